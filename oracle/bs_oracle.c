/*
 * bs_oracle.c -- CPU oracle for the BigSmall bf16 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see bs_oracle.h).  This file restates, in plain
 * C, the algorithms of the reference's CPU codecs so that tests can check
 * the CUDA path byte-for-byte, and so that bench.py can time the
 * reference's fastest CPU decoder on the GPU box's host cores (the
 * reference itself is Python/Numba and cannot travel there).
 *
 * Each function cites the reference lines it follows.  The reference's
 * behaviour on valid streams is reproduced exactly, including its quirks
 * (rans.decode_stream zero-pads an odd trailing byte, numba_rans pads the
 * data to an even length).  Where the reference would read out of bounds
 * or leave memory uninitialised on malformed input, this oracle returns an
 * error code instead.
 */
#include "bs_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define RANS_L (1u << 16)

/* ------------------------------------------------------------------------ */
/* little-endian helpers                                                     */
/* ------------------------------------------------------------------------ */
static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline uint64_t rd64(const uint8_t *p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }
static inline void wr16(uint8_t *p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static inline void wr32(uint8_t *p, uint32_t v) {
    p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}
static inline void wr64(uint8_t *p, uint64_t v) { wr32(p, (uint32_t)v); wr32(p + 4, (uint32_t)(v >> 32)); }

/* bounded byte writer */
typedef struct { uint8_t *p; int64_t len, cap; int err; } bw_t;
static inline void bw_bytes(bw_t *w, const void *src, int64_t n) {
    if (w->err) return;
    if (w->len + n > w->cap) { w->err = 1; return; }
    if (n) memcpy(w->p + w->len, src, (size_t)n);
    w->len += n;
}
static inline void bw_u8(bw_t *w, uint32_t v) { uint8_t b = (uint8_t)v; bw_bytes(w, &b, 1); }
static inline void bw_u16(bw_t *w, uint32_t v) { uint8_t b[2]; wr16(b, v); bw_bytes(w, b, 2); }
static inline void bw_u32(bw_t *w, uint32_t v) { uint8_t b[4]; wr32(b, v); bw_bytes(w, b, 4); }

/* bounded byte reader (Python io.BytesIO + struct.unpack raise on short
 * reads for fixed-size fields; a short `read(n)` of a payload is clamped) */
typedef struct { const uint8_t *p; int64_t len, pos; int err; } br_t;
static inline uint32_t br_u8(br_t *r) { if (r->pos + 1 > r->len) { r->err = 1; return 0; } return r->p[r->pos++]; }
static inline uint32_t br_u16(br_t *r) { if (r->pos + 2 > r->len) { r->err = 1; return 0; } uint32_t v = rd16(r->p + r->pos); r->pos += 2; return v; }
static inline uint32_t br_u32(br_t *r) { if (r->pos + 4 > r->len) { r->err = 1; return 0; } uint32_t v = rd32(r->p + r->pos); r->pos += 4; return v; }
/* clamped payload read: returns pointer and actual length (like BytesIO.read) */
static inline const uint8_t *br_take(br_t *r, int64_t n, int64_t *got) {
    int64_t avail = r->len - r->pos;
    if (avail < 0) avail = 0;
    int64_t k = n < avail ? n : avail;
    const uint8_t *q = r->p + r->pos;
    r->pos += k;
    *got = k;
    return q;
}
/* strict array read: fails if short (np.frombuffer on a short read would
 * produce a shorter array and a later shape error) */
static inline const uint8_t *br_need(br_t *r, int64_t n) {
    if (n < 0 || r->pos + n > r->len) { r->err = 1; return NULL; }
    const uint8_t *q = r->p + r->pos;
    r->pos += n;
    return q;
}

static int ilog2_pow2(uint32_t M) {
    if (M == 0 || (M & (M - 1))) return -1;
    int k = 0;
    while ((1u << k) != M) k++;
    return k;
}

/* ======================================================================== */
/* rans.py                                                                   */
/* ======================================================================== */

/* stable argsort of -scaled: descending by value, ties by ascending index */
static const int64_t *g_sort_keys;
static int cmp_desc_stable(const void *a, const void *b) {
    int ia = *(const int *)a, ib = *(const int *)b;
    int64_t va = g_sort_keys[ia], vb = g_sort_keys[ib];
    if (va != vb) return va > vb ? -1 : 1;
    return ia - ib;
}

/* bigsmall/codecs/rans.py:34-92 quantise_frequencies (numba_rans.py:45-85 is
 * the same algorithm).  Not thread-safe (qsort comparator state). */
static pthread_mutex_t g_sort_mu = PTHREAD_MUTEX_INITIALIZER;
int bso_quantise_ref(const int64_t *counts, int alphabet, uint32_t M, uint32_t *freqs) {
    int n_nz = 0;
    int64_t total = 0;
    for (int i = 0; i < alphabet; i++) if (counts[i] > 0) { n_nz++; total += counts[i]; }
    if (n_nz == 0) {
        memset(freqs, 0, sizeof(uint32_t) * (size_t)alphabet);
        freqs[0] = M;
        return BSO_OK;
    }
    if ((uint32_t)n_nz > M) return BSO_E_ARG;
    int64_t *scaled = (int64_t *)malloc(sizeof(int64_t) * (size_t)alphabet);
    int *order = (int *)malloc(sizeof(int) * (size_t)alphabet);
    if (!scaled || !order) { free(scaled); free(order); return BSO_E_NOMEM; }
    int64_t sum = 0;
    for (int i = 0; i < alphabet; i++) {
        int64_t v = counts[i] > 0 ? (counts[i] * (int64_t)M) / total : 0;
        if (counts[i] > 0 && v < 1) v = 1;
        scaled[i] = v;
        sum += v;
    }
    int64_t diff = (int64_t)M - sum;
    int rc = BSO_OK;
    if (diff != 0) {
        for (int i = 0; i < alphabet; i++) order[i] = i;
        pthread_mutex_lock(&g_sort_mu);
        g_sort_keys = scaled;
        qsort(order, (size_t)alphabet, sizeof(int), cmp_desc_stable);
        pthread_mutex_unlock(&g_sort_mu);
        if (diff > 0) {
            int64_t i = 0;
            while (diff > 0) { scaled[order[i % alphabet]] += 1; diff--; i++; }
        } else {
            int64_t i = 0;
            while (diff < 0) {
                int j = order[i % alphabet];
                if (scaled[j] > 1) { scaled[j] -= 1; diff++; }
                i++;
                if (i > 100 * (int64_t)alphabet) { rc = BSO_E_ARG; break; }
            }
        }
    }
    for (int i = 0; i < alphabet; i++) freqs[i] = (uint32_t)scaled[i];
    free(scaled);
    free(order);
    return rc;
}

static void cum_excl(const uint32_t *freqs, int alphabet, uint32_t *cum) {
    uint32_t c = 0;
    for (int i = 0; i < alphabet; i++) { cum[i] = c; c += freqs[i]; }
}

/* bigsmall/codecs/rans.py:115-162 encode_stream.  Output layout:
 * [u32 final state][u16 renorm words in decode order]. */
int64_t bso_rans_encode(const int32_t *syms, int64_t n, const uint32_t *freqs,
                        int alphabet, uint32_t M, uint8_t *out, int64_t cap) {
    if (n == 0) {
        if (cap < 4) return BSO_E_CAP;
        wr32(out, RANS_L);
        return 4;
    }
    uint32_t *cum = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)alphabet);
    uint16_t *buf = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(n + 1));
    if (!cum || !buf) { free(cum); free(buf); return BSO_E_NOMEM; }
    cum_excl(freqs, alphabet, cum);
    uint64_t state = RANS_L;
    int64_t cnt = 0;
    const uint64_t smax_over_m = (1ull << 32) / M;
    int rc = 0;
    for (int64_t i = n - 1; i >= 0; i--) {
        int32_t s = syms[i];
        if (s < 0 || s >= alphabet || freqs[s] == 0) { rc = BSO_E_ARG; break; }
        uint64_t f = freqs[s], cf = cum[s];
        uint64_t upper = smax_over_m * f;
        while (state >= upper) { buf[cnt++] = (uint16_t)(state & 0xFFFF); state >>= 16; }
        state = (state / f) * M + cf + state % f;
        if (state >= (1ull << 32)) { rc = BSO_E_ARG; break; }
    }
    int64_t need = 4 + 2 * cnt;
    if (rc == 0 && need > cap) rc = BSO_E_CAP;
    if (rc == 0) {
        wr32(out, (uint32_t)state);
        for (int64_t k = 0; k < cnt; k++) wr16(out + 4 + 2 * k, buf[cnt - 1 - k]);
    }
    free(cum);
    free(buf);
    return rc ? rc : need;
}

/* bigsmall/codecs/rans.py:165-207 decode_stream, including the renorm loop's
 * end-of-data behaviour (:196-202): with one byte left the state is shifted
 * by 16 with zero fill and reading stops; with none left reading stops. */
int bso_rans_decode(const uint8_t *data, int64_t len, int64_t n,
                    const uint32_t *freqs, int alphabet, uint32_t M, uint32_t *out) {
    if (n == 0) return BSO_OK;
    if (len < 4) return BSO_E_TRUNC;
    int logm = ilog2_pow2(M);
    if (logm < 0) return BSO_E_ARG;
    uint32_t *cum = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)alphabet);
    uint16_t *s2s = (uint16_t *)calloc(M, sizeof(uint16_t));   /* rans.py:102-112 */
    if (!cum || !s2s) { free(cum); free(s2s); return BSO_E_NOMEM; }
    cum_excl(freqs, alphabet, cum);
    for (int s = 0; s < alphabet; s++)
        for (uint32_t j = 0; j < freqs[s] && cum[s] + j < M; j++) s2s[cum[s] + j] = (uint16_t)s;
    uint64_t state = rd32(data);
    int64_t pos = 4;
    for (int64_t i = 0; i < n; i++) {
        uint32_t slot = (uint32_t)(state & (M - 1));
        uint32_t s = s2s[slot];
        out[i] = s;
        uint64_t f = freqs[s], cf = cum[s];
        state = f * (state >> logm) + slot - cf;
        while (state < RANS_L && pos < len) {
            if (pos + 2 > len) { state <<= 16; pos = len; break; }
            state = (state << 16) | rd16(data + pos);
            pos += 2;
        }
    }
    free(cum);
    free(s2s);
    return BSO_OK;
}

/* numba_rans.py:168-217 decode_stream: the data is padded to an even length
 * and read as u16; the state is u16[0] | u16[1] << 16; renorm reads while
 * state < L and words remain.  single_kernel.py:160-190 is the same loop. */
static int nr_decode(const uint8_t *data, int64_t len, int64_t n, const uint32_t *freqs,
                     int alphabet, int prec, uint32_t *out) {
    if (n == 0) return BSO_OK;
    if (len < 4) return BSO_E_TRUNC;
    uint32_t M = 1u << prec;
    uint32_t *cum = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)alphabet);
    uint32_t *s2s = (uint32_t *)calloc(M, sizeof(uint32_t));
    if (!cum || !s2s) { free(cum); free(s2s); return BSO_E_NOMEM; }
    cum_excl(freqs, alphabet, cum);
    for (int s = 0; s < alphabet; s++)
        for (uint32_t j = 0; j < freqs[s] && cum[s] + j < M; j++) s2s[cum[s] + j] = (uint32_t)s;
    int64_t nwords = (len + 1) / 2;    /* odd length padded with a zero byte */
    #define NRW(k) ((2 * (k) + 1 < len) ? rd16(data + 2 * (k)) : (uint16_t)data[2 * (k)])
    uint64_t state = (uint64_t)NRW(0) | ((uint64_t)NRW(1) << 16);
    int64_t pos = 2;
    for (int64_t i = 0; i < n; i++) {
        uint32_t slot = (uint32_t)(state & (M - 1));
        uint32_t s = s2s[slot];
        out[i] = s;
        uint64_t f = freqs[s], cf = cum[s];
        state = f * (state >> prec) + slot - cf;
        while (state < RANS_L && pos < nwords) { state = (state << 16) | NRW(pos); pos++; }
    }
    #undef NRW
    free(cum);
    free(s2s);
    return BSO_OK;
}

/* ======================================================================== */
/* bf16_parallel_v1 (bigsmall/codecs/bf16_parallel.py)                      */
/* ======================================================================== */
#define PAR_PREC_SE 12
#define PAR_PREC_M 10
#define PAR_M_SE (1u << PAR_PREC_SE)
#define PAR_M_M (1u << PAR_PREC_M)

int64_t bso_par_bound(int64_t n, int n_streams) {
    int64_t ns = n_streams < 1 ? 1 : n_streams;
    /* header <= 4+4+2+2+2+2+512*6+4+256*2+256*(1+128*5); per stream framing
     * <= 12 + 256*(2+8+4); symbols cost <= 2 bytes each in the worst case */
    return 8192 + 256 * 650 + (ns + 1) * 4 + ns * (16 + 256 * 20) + 4 * n + 64;
}

/* bigsmall/codecs/bf16_parallel.py:186-259 encode */
int64_t bso_par_encode(const uint16_t *w, int64_t n, int n_streams, uint8_t *out, int64_t cap) {
    if (n == 0) return 0;
    int64_t ns = n_streams;
    if (ns > n) ns = n;
    if (ns < 1) ns = 1;
    if (ns > 65535 || n > 0xFFFFFFFFll) return BSO_E_ARG;
    int rc = 0;
    /* _build_shared_freqs :77-103 */
    int64_t se_counts[512] = {0}, exp_counts[256] = {0};
    static const int A_M = 128;
    int64_t (*mc)[128] = calloc(256, sizeof(*mc));
    uint32_t se_freqs[512];
    uint32_t (*mf)[128] = calloc(256, sizeof(*mf));
    if (!mc || !mf) { free(mc); free(mf); return BSO_E_NOMEM; }
    for (int64_t i = 0; i < n; i++) {
        uint32_t v = w[i], e = (v >> 7) & 0xFF;
        se_counts[((v >> 15) << 8) | e]++;
        exp_counts[e]++;
        mc[e][v & 0x7F]++;
    }
    rc = bso_quantise_ref(se_counts, 512, PAR_M_SE, se_freqs);
    for (int e = 0; e < 256 && !rc; e++)
        if (exp_counts[e]) rc = bso_quantise_ref(mc[e], A_M, PAR_M_M, mf[e]);
    if (rc) { free(mc); free(mf); return rc; }
    bw_t bw = {out, 0, cap, 0};
    /* _pack_header :106-135 */
    bw_bytes(&bw, "PAR1", 4);
    bw_u32(&bw, (uint32_t)n);
    bw_u16(&bw, (uint32_t)ns);
    bw_u16(&bw, PAR_PREC_SE);
    bw_u16(&bw, PAR_PREC_M);
    int n_se_nz = 0;
    for (int i = 0; i < 512; i++) n_se_nz += se_freqs[i] > 0;
    bw_u16(&bw, (uint32_t)n_se_nz);
    for (int i = 0; i < 512; i++) if (se_freqs[i]) bw_u16(&bw, (uint32_t)i);
    for (int i = 0; i < 512; i++) if (se_freqs[i]) bw_u32(&bw, se_freqs[i]);
    int n_exps = 0;
    for (int e = 0; e < 256; e++) n_exps += exp_counts[e] > 0;
    bw_u32(&bw, (uint32_t)n_exps);
    for (int e = 0; e < 256; e++) if (exp_counts[e]) bw_u16(&bw, (uint32_t)e);
    for (int e = 0; e < 256; e++) {
        if (!exp_counts[e]) continue;
        int nz = 0;
        for (int m = 0; m < 128; m++) nz += mf[e][m] > 0;
        bw_u8(&bw, (uint32_t)nz);
        for (int m = 0; m < 128; m++) if (mf[e][m]) bw_u8(&bw, (uint32_t)m);
        for (int m = 0; m < 128; m++) if (mf[e][m]) bw_u32(&bw, mf[e][m]);
    }
    int64_t off_pos = bw.len;
    for (int64_t k = 0; k <= ns; k++) bw_u32(&bw, 0);   /* patched below */
    int64_t payload_start = bw.len;
    int64_t slice_cap = n / ns + 1;
    int32_t *se_s = (int32_t *)malloc(sizeof(int32_t) * (size_t)slice_cap);
    int32_t *bucket = (int32_t *)malloc(sizeof(int32_t) * (size_t)slice_cap);
    uint8_t *tmp = (uint8_t *)malloc((size_t)(4 + 2 * slice_cap + 16));
    if (!se_s || !bucket || !tmp) rc = BSO_E_NOMEM;
    for (int64_t k = 0; k < ns && !rc && !bw.err; k++) {
        wr32(out + off_pos + 4 * k, (uint32_t)(bw.len - payload_start));
        int64_t cnt = 0;
        int64_t ecount[256] = {0};
        for (int64_t i = k; i < n; i += ns) {
            uint32_t v = w[i];
            se_s[cnt++] = (int32_t)(((v >> 15) << 8) | ((v >> 7) & 0xFF));
            ecount[(v >> 7) & 0xFF]++;
        }
        /* SE rANS stream :218-221 */
        int64_t L1 = bso_rans_encode(se_s, cnt, se_freqs, 512, PAR_M_SE, tmp, 4 + 2 * slice_cap + 16);
        if (L1 < 0) { rc = (int)L1; break; }
        bw_u32(&bw, (uint32_t)L1);
        bw_bytes(&bw, tmp, L1);
        /* mantissa buckets in ascending exp, stable order :223-242 */
        int nze = 0;
        for (int e = 0; e < 256; e++) nze += ecount[e] > 0;
        bw_u32(&bw, (uint32_t)nze);
        for (int e = 0; e < 256; e++) if (ecount[e]) bw_u16(&bw, (uint32_t)e);
        for (int e = 0; e < 256 && !rc; e++) {
            if (!ecount[e]) continue;
            int64_t bc = 0;
            for (int64_t i = k; i < n; i += ns)
                if (((w[i] >> 7) & 0xFF) == (uint32_t)e) bucket[bc++] = (int32_t)(w[i] & 0x7F);
            int64_t L2 = bso_rans_encode(bucket, bc, mf[e], 128, PAR_M_M, tmp, 4 + 2 * slice_cap + 16);
            if (L2 < 0) { rc = (int)L2; break; }
            bw_u32(&bw, (uint32_t)bc);
            bw_u32(&bw, (uint32_t)L2);
            bw_bytes(&bw, tmp, L2);
        }
    }
    if (!rc && !bw.err) wr32(out + off_pos + 4 * ns, (uint32_t)(bw.len - payload_start));
    free(se_s); free(bucket); free(tmp); free(mc); free(mf);
    if (rc) return rc;
    if (bw.err) return BSO_E_CAP;
    return bw.len;
}

/* bigsmall/codecs/bf16_parallel.py:138-183 _unpack_header + :262-352 decode */
int bso_par_decode(const uint8_t *blob, int64_t len, int64_t n_weights, uint16_t *out) {
    if (n_weights == 0 || len == 0) return BSO_OK;
    br_t r = {blob, len, 0, 0};
    const uint8_t *mg = br_need(&r, 4);
    if (!mg) return BSO_E_TRUNC;
    if (memcmp(mg, "PAR1", 4) != 0) return BSO_E_MAGIC;
    int64_t n = br_u32(&r);
    int64_t ns = br_u16(&r);
    uint32_t p_se = br_u16(&r), p_m = br_u16(&r);
    if (r.err) return BSO_E_TRUNC;
    if (p_se != PAR_PREC_SE || p_m != PAR_PREC_M) return BSO_E_PREC;
    uint32_t n_se_nz = br_u16(&r);
    const uint8_t *idx = br_need(&r, 2 * (int64_t)n_se_nz);
    const uint8_t *fr = br_need(&r, 4 * (int64_t)n_se_nz);
    if (r.err) return BSO_E_TRUNC;
    uint32_t se_freqs[512] = {0};
    for (uint32_t i = 0; i < n_se_nz; i++) {
        uint32_t s = rd16(idx + 2 * i);
        if (s >= 512) return BSO_E_CORRUPT;
        se_freqs[s] = rd32(fr + 4 * i);
    }
    uint32_t n_exps = br_u32(&r);
    const uint8_t *ex = br_need(&r, 2 * (int64_t)n_exps);
    if (r.err) return BSO_E_TRUNC;
    uint32_t (*mf)[128] = calloc(256, sizeof(*mf));
    uint8_t has_mf[256] = {0};
    if (!mf) return BSO_E_NOMEM;
    int rc = 0;
    for (uint32_t q = 0; q < n_exps && !rc; q++) {
        uint32_t ev = rd16(ex + 2 * q);
        uint32_t nzc = br_u8(&r);
        const uint8_t *nz = br_need(&r, nzc);
        const uint8_t *nzf = br_need(&r, 4 * (int64_t)nzc);
        if (r.err) { rc = BSO_E_TRUNC; break; }
        if (ev >= 256) { rc = BSO_E_CORRUPT; break; }
        memset(mf[ev], 0, sizeof(mf[ev]));
        for (uint32_t i = 0; i < nzc; i++) {
            if (nz[i] >= 128) { rc = BSO_E_CORRUPT; break; }
            mf[ev][nz[i]] = rd32(nzf + 4 * i);
        }
        has_mf[ev] = 1;
    }
    if (!rc && n != n_weights) rc = BSO_E_COUNT;
    if (rc) { free(mf); return rc; }
    int64_t header_end = r.pos;
    int64_t n_off = ns + 1;
    if (header_end + 4 * n_off > len) { free(mf); return BSO_E_TRUNC; }
    const uint8_t *offt = blob + header_end;
    int64_t payload_start = header_end + 4 * n_off;
    int64_t maxs = ns ? (n + ns - 1) / ns : 0;
    uint32_t *se_sl = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(maxs + 1));
    uint32_t *msym = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(maxs + 1));
    uint16_t *msorted = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(maxs + 1));
    uint8_t *filled = (uint8_t *)malloc((size_t)(maxs + 1));
    if (!se_sl || !msym || !msorted || !filled) rc = BSO_E_NOMEM;
    for (int64_t k = 0; k < ns && !rc; k++) {
        int64_t nin = k < n ? (n - 1 - k) / ns + 1 : 0;
        if (nin == 0) continue;
        /* python slicing of blob[ps+off[k] : ps+off[k+1]] clamps */
        int64_t a = payload_start + rd32(offt + 4 * k), b = payload_start + rd32(offt + 4 * (k + 1));
        if (a > len) a = len;
        if (b > len) b = len;
        if (b < a) b = a;
        br_t s = {blob + a, b - a, 0, 0};
        uint32_t se_len = br_u32(&s);
        if (s.err) { rc = BSO_E_TRUNC; break; }
        int64_t got;
        const uint8_t *se_blob = br_take(&s, se_len, &got);
        rc = bso_rans_decode(se_blob, got, nin, se_freqs, 512, PAR_M_SE, se_sl);
        if (rc) break;
        int64_t bstart[257] = {0};
        for (int64_t i = 0; i < nin; i++) bstart[(se_sl[i] & 0xFF) + 1]++;
        for (int e = 0; e < 256; e++) bstart[e + 1] += bstart[e];
        uint32_t nze = br_u32(&s);
        const uint8_t *sx = br_need(&s, 2 * (int64_t)nze);
        if (s.err) { rc = BSO_E_TRUNC; break; }
        memset(filled, 0, (size_t)nin);
        for (uint32_t q = 0; q < nze && !rc; q++) {
            uint32_t ev = rd16(sx + 2 * q);
            uint32_t count = br_u32(&s), blen = br_u32(&s);
            if (s.err) { rc = BSO_E_TRUNC; break; }
            const uint8_t *mb = br_take(&s, blen, &got);
            if (ev >= 256 || !has_mf[ev]) { rc = BSO_E_CORRUPT; break; }
            if ((int64_t)count != bstart[ev + 1] - bstart[ev]) { rc = BSO_E_CORRUPT; break; }
            rc = bso_rans_decode(mb, got, count, mf[ev], 128, PAR_M_M, msym);
            for (uint32_t i = 0; i < count && !rc; i++) {
                msorted[bstart[ev] + i] = (uint16_t)msym[i];
                filled[bstart[ev] + i] = 1;
            }
        }
        if (rc) break;
        for (int64_t i = 0; i < nin; i++) if (!filled[i]) { rc = BSO_E_CORRUPT; break; }
        if (rc) break;
        /* un-sort (stable argsort inverse, :328-344) and merge (:349-352) */
        int64_t cur[256];
        for (int e = 0; e < 256; e++) cur[e] = bstart[e];
        for (int64_t i = 0; i < nin; i++) {
            uint32_t se = se_sl[i], e = se & 0xFF;
            uint32_t m = msorted[cur[e]++];
            out[k + i * ns] = (uint16_t)((((se >> 8) & 1) << 15) | (e << 7) | m);
        }
    }
    free(se_sl); free(msym); free(msorted); free(filled); free(mf);
    return rc;
}

/* ======================================================================== */
/* bf16_se_single_kernel (bigsmall/codecs/single_kernel.py)                  */
/* ======================================================================== */

/* single_kernel.py:54-110 _quantise_inplace (argmax based; differs from
 * rans.quantise_frequencies) */
static void sk_quantise(const int64_t *counts, int alphabet, int64_t M, uint32_t *out) {
    int n_nz = 0;
    int64_t total = 0;
    for (int i = 0; i < alphabet; i++) if (counts[i] > 0) { n_nz++; total += counts[i]; }
    if (n_nz == 0) {
        for (int i = 0; i < alphabet; i++) out[i] = 0;
        out[0] = (uint32_t)M;
        return;
    }
    int64_t s = 0;
    for (int i = 0; i < alphabet; i++) {
        if (counts[i] > 0) {
            int64_t v = (counts[i] * M) / total;
            if (v < 1) v = 1;
            out[i] = (uint32_t)v;
            s += v;
        } else out[i] = 0;
    }
    int64_t diff = M - s;
    if (diff > 0) {
        while (diff > 0) {
            int best = 0; uint32_t bv = 0;
            for (int i = 0; i < alphabet; i++) if (out[i] > bv) { bv = out[i]; best = i; }
            out[best] += 1;
            diff--;
        }
    } else if (diff < 0) {
        int64_t guard = 0;
        while (diff < 0 && guard < 50 * (int64_t)alphabet) {
            int best = 0; uint32_t bv = 0;
            for (int i = 0; i < alphabet; i++) if (out[i] > bv) { bv = out[i]; best = i; }
            if (out[best] > 1) { out[best] -= 1; diff++; } else break;
            guard++;
        }
    }
}

/* single_kernel.py:122-156 _rans_encode_one: returns the number of words;
 * words land in buf in reverse decode order. */
static int64_t sk_encode_one(const uint8_t *sym8, const uint16_t *sym16, int64_t n,
                             const uint32_t *freqs, const uint32_t *cum, int64_t M,
                             uint16_t *buf, uint32_t *final_state) {
    if (n == 0) { *final_state = RANS_L; return 0; }
    uint64_t state = RANS_L, lb = (1ull << 32) / (uint64_t)M;
    int64_t c = 0;
    for (int64_t i = n - 1; i >= 0; i--) {
        uint32_t s = sym8 ? sym8[i] : sym16[i];
        uint64_t f = freqs[s], cf = cum[s];
        uint64_t upper = lb * f;
        while (state >= upper) { buf[c++] = (uint16_t)(state & 0xFFFF); state >>= 16; }
        state = (state / f) * (uint64_t)M + cf + state % f;
    }
    *final_state = (uint32_t)state;
    return c;
}

int64_t bso_sk_bound(int64_t n) { return 4 * n + 64 * 1024; }   /* single_kernel.py:595 */

/* single_kernel.py:194-428 _encode_full_kernel */
int64_t bso_sk_encode(const uint16_t *w, int64_t n, uint8_t *out, int64_t cap) {
    if (n == 0) return 0;
    if (n > 0xFFFFFFFFll) return BSO_E_ARG;
    int64_t se_counts[512] = {0}, exp_counts[256] = {0};
    uint16_t *se = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n);
    uint8_t *msorted = (uint8_t *)malloc((size_t)n);
    uint16_t *scratch = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(n + 64));
    uint16_t *bscratch = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(n + 64));
    if (!se || !msorted || !scratch || !bscratch) {
        free(se); free(msorted); free(scratch); free(bscratch); return BSO_E_NOMEM;
    }
    for (int64_t i = 0; i < n; i++) {
        uint32_t v = w[i], e = (v >> 7) & 0xFF;
        se[i] = (uint16_t)(((v >> 15) << 8) | e);
        se_counts[se[i]]++;
        exp_counts[e]++;
    }
    uint32_t se_freqs[512], se_cum[512];
    sk_quantise(se_counts, 512, 4096, se_freqs);
    se_cum[0] = 0;
    for (int i = 1; i < 512; i++) se_cum[i] = se_cum[i - 1] + se_freqs[i - 1];
    int64_t bstart[257];
    bstart[0] = 0;
    for (int i = 0; i < 256; i++) bstart[i + 1] = bstart[i] + exp_counts[i];
    int64_t cur[256];
    for (int i = 0; i < 256; i++) cur[i] = bstart[i];
    for (int64_t i = 0; i < n; i++) { uint32_t e = (w[i] >> 7) & 0xFF; msorted[cur[e]++] = (uint8_t)(w[i] & 0x7F); }
    bw_t bw = {out, 0, cap, 0};
    bw_u32(&bw, (uint32_t)n);
    int n_se_nz = 0;
    for (int i = 0; i < 512; i++) n_se_nz += se_freqs[i] > 0;
    bw_u16(&bw, (uint32_t)n_se_nz);
    for (int i = 0; i < 512; i++) if (se_freqs[i]) bw_u16(&bw, (uint32_t)i);
    for (int i = 0; i < 512; i++) if (se_freqs[i]) bw_u32(&bw, se_freqs[i]);
    uint32_t st;
    int64_t c = sk_encode_one(NULL, se, n, se_freqs, se_cum, 4096, scratch, &st);
    bw_u32(&bw, st);
    bw_u32(&bw, (uint32_t)c);
    for (int64_t k = c - 1; k >= 0; k--) bw_u16(&bw, scratch[k]);
    int n_nz_exps = 0;
    for (int e = 0; e < 256; e++) n_nz_exps += exp_counts[e] > 0;
    bw_u32(&bw, (uint32_t)n_nz_exps);
    for (int e = 0; e < 256; e++) {
        if (!exp_counts[e]) continue;
        int64_t bc[128] = {0};
        for (int64_t i = bstart[e]; i < bstart[e + 1]; i++) bc[msorted[i]]++;
        uint32_t mf[128], mcum[128];
        sk_quantise(bc, 128, 1024, mf);
        mcum[0] = 0;
        for (int i = 1; i < 128; i++) mcum[i] = mcum[i - 1] + mf[i - 1];
        int64_t bs = bstart[e + 1] - bstart[e];
        int64_t cc = sk_encode_one(msorted + bstart[e], NULL, bs, mf, mcum, 1024, bscratch, &st);
        bw_u16(&bw, (uint32_t)e);
        int mnz = 0;
        for (int i = 0; i < 128; i++) mnz += mf[i] > 0;
        bw_u8(&bw, (uint32_t)mnz);
        for (int i = 0; i < 128; i++) if (mf[i]) bw_u8(&bw, (uint32_t)i);
        for (int i = 0; i < 128; i++) if (mf[i]) bw_u32(&bw, mf[i]);
        bw_u32(&bw, st);
        bw_u32(&bw, (uint32_t)bs);
        bw_u32(&bw, (uint32_t)cc);
        for (int64_t k = cc - 1; k >= 0; k--) bw_u16(&bw, bscratch[k]);
    }
    free(se); free(msorted); free(scratch); free(bscratch);
    return bw.err ? BSO_E_CAP : bw.len;
}

/* build a u32 slot->(sym | freq<<..) free form: separate arrays are fine */
static int sk_tables(const uint32_t *freqs, int alphabet, uint32_t M, uint32_t *cum, uint32_t *s2s) {
    uint64_t c = 0;
    for (int i = 0; i < alphabet; i++) { cum[i] = (uint32_t)c; c += freqs[i]; }
    if (c != M) return BSO_E_CORRUPT;   /* the reference would leave slots uninitialised */
    for (int s = 0; s < alphabet; s++)
        for (uint32_t j = 0; j < freqs[s]; j++) s2s[cum[s] + j] = (uint32_t)s;
    return BSO_OK;
}

/* single_kernel.py:160-190 _rans_decode_one over an in-blob word array.
 * `words` points at the nc renorm u16s; the state comes separately. */
static inline void sk_decode_one(uint32_t state0, const uint8_t *words, int64_t nc, int64_t n,
                                 const uint32_t *freqs, const uint32_t *cum, const uint32_t *s2s,
                                 int prec, uint32_t *out32, uint8_t *out8) {
    uint32_t mask = (1u << prec) - 1;
    uint64_t state = state0;
    int64_t pos = 0;
    for (int64_t i = 0; i < n; i++) {
        uint32_t slot = (uint32_t)(state & mask);
        uint32_t s = s2s[slot];
        if (out32) out32[i] = s; else out8[i] = (uint8_t)s;
        state = (uint64_t)freqs[s] * (state >> prec) + slot - cum[s];
        while (state < RANS_L && pos < nc) { state = (state << 16) | rd16(words + 2 * pos); pos++; }
    }
}

/* single_kernel.py:432-580 _decode_full_kernel (+ :603-613 decode) */
int bso_sk_decode(const uint8_t *blob, int64_t len, int64_t n_weights, uint16_t *out) {
    if (n_weights == 0 || len == 0) return BSO_OK;
    br_t r = {blob, len, 0, 0};
    int64_t n = br_u32(&r);
    if (r.err) return BSO_E_TRUNC;
    if (n != n_weights) return BSO_E_COUNT;   /* the reference silently returns (:445-446) */
    uint32_t n_se_nz = br_u16(&r);
    const uint8_t *idx = br_need(&r, 2 * (int64_t)n_se_nz);
    const uint8_t *fr = br_need(&r, 4 * (int64_t)n_se_nz);
    if (r.err) return BSO_E_TRUNC;
    uint32_t se_freqs[512] = {0}, se_cum[512];
    for (uint32_t i = 0; i < n_se_nz; i++) {
        uint32_t s = rd16(idx + 2 * i);
        if (s >= 512) return BSO_E_CORRUPT;
        se_freqs[s] = rd32(fr + 4 * i);
    }
    uint32_t *se_s2s = (uint32_t *)malloc(sizeof(uint32_t) * 4096);
    uint32_t *se_dec = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n);
    uint8_t *msorted = (uint8_t *)malloc((size_t)n);
    uint8_t *bucket = (uint8_t *)malloc((size_t)n);
    int rc = (!se_s2s || !se_dec || !msorted || !bucket) ? BSO_E_NOMEM : 0;
    if (!rc) rc = sk_tables(se_freqs, 512, 4096, se_cum, se_s2s);
    uint32_t st = 0, nc = 0;
    const uint8_t *wd = NULL;
    if (!rc) {
        st = br_u32(&r);
        nc = br_u32(&r);
        wd = br_need(&r, 2 * (int64_t)nc);
        if (r.err) rc = BSO_E_TRUNC;
    }
    if (!rc) sk_decode_one(st, wd, nc, n, se_freqs, se_cum, se_s2s, 12, se_dec, NULL);
    int64_t bstart[257] = {0};
    if (!rc) {
        for (int64_t i = 0; i < n; i++) bstart[(se_dec[i] & 0xFF) + 1]++;
        for (int e = 0; e < 256; e++) bstart[e + 1] += bstart[e];
    }
    uint32_t n_nz_exps = rc ? 0 : br_u32(&r);
    if (r.err) rc = BSO_E_TRUNC;
    uint8_t seen[256] = {0};
    for (uint32_t b = 0; b < n_nz_exps && !rc; b++) {
        uint32_t e = br_u16(&r);
        uint32_t mnz = br_u8(&r);
        const uint8_t *nz = br_need(&r, mnz);
        const uint8_t *nzf = br_need(&r, 4 * (int64_t)mnz);
        if (r.err) { rc = BSO_E_TRUNC; break; }
        if (e >= 256) { rc = BSO_E_CORRUPT; break; }
        uint32_t mf[128] = {0}, mcum[128], ms2s[1024];
        for (uint32_t i = 0; i < mnz; i++) {
            if (nz[i] >= 128) { rc = BSO_E_CORRUPT; break; }
            mf[nz[i]] = rd32(nzf + 4 * i);
        }
        if (rc) break;
        rc = sk_tables(mf, 128, 1024, mcum, ms2s);
        if (rc) break;
        uint32_t mst = br_u32(&r), bsize = br_u32(&r), mnc = br_u32(&r);
        const uint8_t *mw = br_need(&r, 2 * (int64_t)mnc);
        if (r.err) { rc = BSO_E_TRUNC; break; }
        if ((int64_t)bsize != bstart[e + 1] - bstart[e]) { rc = BSO_E_CORRUPT; break; }
        sk_decode_one(mst, mw, mnc, bsize, mf, mcum, ms2s, 10, NULL, msorted + bstart[e]);
        seen[e] = 1;
    }
    for (int e = 0; e < 256 && !rc; e++)
        if (bstart[e + 1] > bstart[e] && !seen[e]) rc = BSO_E_CORRUPT;
    if (!rc) {
        /* un-sort via cursor walk (:570-580) */
        int64_t cur[256];
        for (int e = 0; e < 256; e++) cur[e] = bstart[e];
        for (int64_t i = 0; i < n; i++) {
            uint32_t se = se_dec[i], e = se & 0xFF;
            out[i] = (uint16_t)((((se >> 8) & 1) << 15) | (e << 7) | msorted[cur[e]++]);
        }
    }
    free(se_s2s); free(se_dec); free(msorted); free(bucket);
    return rc;
}

/* ======================================================================== */
/* bf16_se_tans (bigsmall/codecs/bf16_tans.py + numba_rans.py)               */
/* ======================================================================== */
int64_t bso_tans_bound(int64_t n) { return 4 * n + 256 * 1024; }

/* bigsmall/codecs/bf16_tans.py:289-339 encode */
int64_t bso_tans_encode(const uint16_t *w, int64_t n, uint8_t *out, int64_t cap) {
    if (n == 0) return 0;
    if (n > 0xFFFFFFFFll) return BSO_E_ARG;
    int64_t se_counts[512] = {0}, exp_counts[256] = {0};
    int32_t *syms = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    uint8_t *tmp = (uint8_t *)malloc((size_t)(4 + 2 * n + 16));
    uint8_t *msorted = (uint8_t *)malloc((size_t)n);
    if (!syms || !tmp || !msorted) { free(syms); free(tmp); free(msorted); return BSO_E_NOMEM; }
    for (int64_t i = 0; i < n; i++) {
        uint32_t v = w[i], e = (v >> 7) & 0xFF;
        syms[i] = (int32_t)(((v >> 15) << 8) | e);
        se_counts[syms[i]]++;
        exp_counts[e]++;
    }
    uint32_t se_freqs[512];
    int rc = bso_quantise_ref(se_counts, 512, 4096, se_freqs);
    int64_t se_len = rc ? 0 : bso_rans_encode(syms, n, se_freqs, 512, 4096, tmp, 4 + 2 * n + 16);
    if (se_len < 0) rc = (int)se_len;
    bw_t bw = {out, 0, cap, 0};
    if (!rc) {
        bw_u32(&bw, (uint32_t)n);
        int nz = 0;
        for (int i = 0; i < 512; i++) nz += se_freqs[i] > 0;
        bw_u16(&bw, (uint32_t)nz);
        for (int i = 0; i < 512; i++) if (se_freqs[i]) bw_u16(&bw, (uint32_t)i);
        for (int i = 0; i < 512; i++) if (se_freqs[i]) bw_u32(&bw, se_freqs[i]);
        bw_u32(&bw, (uint32_t)se_len);
        bw_bytes(&bw, tmp, se_len);
    }
    int64_t mlen_pos = bw.len;
    if (!rc) {
        bw_u32(&bw, 0);   /* m_blob length, patched */
        /* stable argsort of exp == counting sort */
        int64_t bstart[257];
        bstart[0] = 0;
        for (int i = 0; i < 256; i++) bstart[i + 1] = bstart[i] + exp_counts[i];
        int64_t cur[256];
        for (int i = 0; i < 256; i++) cur[i] = bstart[i];
        for (int64_t i = 0; i < n; i++) { uint32_t e = (w[i] >> 7) & 0xFF; msorted[cur[e]++] = (uint8_t)(w[i] & 0x7F); }
        int ne = 0;
        for (int e = 0; e < 256; e++) ne += exp_counts[e] > 0;
        bw_u32(&bw, (uint32_t)ne);
        for (int e = 0; e < 256; e++) if (exp_counts[e]) bw_u16(&bw, (uint32_t)e);
        for (int e = 0; e < 256 && !rc; e++) {
            if (!exp_counts[e]) continue;
            int64_t bs = bstart[e], be = bstart[e + 1];
            int64_t bc[128] = {0};
            for (int64_t i = bs; i < be; i++) { bc[msorted[i]]++; syms[i - bs] = msorted[i]; }
            uint32_t mf[128];
            rc = bso_quantise_ref(bc, 128, 1024, mf);
            if (rc) break;
            int64_t cl = bso_rans_encode(syms, be - bs, mf, 128, 1024, tmp, 4 + 2 * n + 16);
            if (cl < 0) { rc = (int)cl; break; }
            int mnz = 0;
            for (int i = 0; i < 128; i++) mnz += mf[i] > 0;
            bw_u32(&bw, (uint32_t)(be - bs));
            bw_u8(&bw, (uint32_t)mnz);
            for (int i = 0; i < 128; i++) if (mf[i]) bw_u8(&bw, (uint32_t)i);
            for (int i = 0; i < 128; i++) if (mf[i]) bw_u32(&bw, mf[i]);
            bw_u32(&bw, (uint32_t)cl);
            bw_bytes(&bw, tmp, cl);
        }
    }
    if (!rc && !bw.err) wr32(out + mlen_pos, (uint32_t)(bw.len - mlen_pos - 4));
    free(syms); free(tmp); free(msorted);
    if (rc) return rc;
    return bw.err ? BSO_E_CAP : bw.len;
}

/* bigsmall/codecs/bf16_tans.py:342-388 decode */
int bso_tans_decode(const uint8_t *blob, int64_t len, int64_t n_weights, uint16_t *out) {
    if (n_weights == 0 || len == 0) return BSO_OK;
    br_t r = {blob, len, 0, 0};
    int64_t n = br_u32(&r);
    if (r.err) return BSO_E_TRUNC;
    if (n != n_weights) return BSO_E_COUNT;
    uint32_t se_nz = br_u16(&r);
    const uint8_t *idx = br_need(&r, 2 * (int64_t)se_nz);
    const uint8_t *fr = br_need(&r, 4 * (int64_t)se_nz);
    uint32_t cwl = br_u32(&r);
    if (r.err) return BSO_E_TRUNC;
    int64_t got;
    const uint8_t *cw = br_take(&r, cwl, &got);
    uint32_t se_freqs[512] = {0};
    for (uint32_t i = 0; i < se_nz; i++) {
        uint32_t s = rd16(idx + 2 * i);
        if (s >= 512) return BSO_E_CORRUPT;
        se_freqs[s] = rd32(fr + 4 * i);
    }
    uint32_t *se = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n);
    uint32_t *ms = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n);
    uint8_t *filled = (uint8_t *)calloc((size_t)n, 1);
    int rc = (!se || !ms || !filled) ? BSO_E_NOMEM : 0;
    if (!rc) rc = nr_decode(cw, got, n, se_freqs, 512, 12, se);
    int64_t bstart[257] = {0};
    if (!rc) {
        for (int64_t i = 0; i < n; i++) bstart[(se[i] & 0xFF) + 1]++;
        for (int e = 0; e < 256; e++) bstart[e + 1] += bstart[e];
    }
    uint32_t mbl = rc ? 0 : br_u32(&r);
    if (r.err) rc = BSO_E_TRUNC;
    const uint8_t *mb = rc ? NULL : br_take(&r, mbl, &got);
    br_t m = {mb, got, 0, 0};
    uint32_t ne = rc ? 0 : br_u32(&m);
    const uint8_t *ex = rc ? NULL : br_need(&m, 2 * (int64_t)ne);
    if (!rc && m.err) rc = BSO_E_TRUNC;
    uint16_t *msorted = rc ? NULL : (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n);
    if (!rc && !msorted) rc = BSO_E_NOMEM;
    for (uint32_t q = 0; q < ne && !rc; q++) {
        uint32_t ev = rd16(ex + 2 * q);
        uint32_t nb = br_u32(&m), nnz = br_u8(&m);
        const uint8_t *nz = br_need(&m, nnz);
        const uint8_t *nzf = br_need(&m, 4 * (int64_t)nnz);
        uint32_t cl = br_u32(&m);
        if (m.err) { rc = BSO_E_TRUNC; break; }
        const uint8_t *c2 = br_take(&m, cl, &got);
        if (ev >= 256 || (int64_t)nb != bstart[ev + 1] - bstart[ev]) { rc = BSO_E_CORRUPT; break; }
        uint32_t mf[128] = {0};
        for (uint32_t i = 0; i < nnz; i++) {
            if (nz[i] >= 128) { rc = BSO_E_CORRUPT; break; }
            mf[nz[i]] = rd32(nzf + 4 * i);
        }
        if (rc) break;
        rc = nr_decode(c2, got, nb, mf, 128, 10, ms);
        for (uint32_t i = 0; i < nb && !rc; i++) {
            msorted[bstart[ev] + i] = (uint16_t)ms[i];
            filled[bstart[ev] + i] = 1;
        }
    }
    for (int64_t i = 0; i < n && !rc; i++) if (!filled[i]) rc = BSO_E_CORRUPT;
    if (!rc) {
        int64_t cur[256];
        for (int e = 0; e < 256; e++) cur[e] = bstart[e];
        for (int64_t i = 0; i < n; i++) {
            uint32_t s = se[i], e = s & 0xFF;
            out[i] = (uint16_t)((((s >> 8) & 1) << 15) | (e << 7) | msorted[cur[e]++]);
        }
    }
    free(se); free(ms); free(filled); free(msorted);
    return rc;
}

/* ======================================================================== */
/* bf16_exp_chunked_v1 -- this project's chunked format (no reference       */
/* counterpart).  Layout (little-endian; sections in this fixed order, each  */
/* 16-byte aligned):                                                         */
/*   0   "BSXC"   4 u16 version (1, or 2 with groups)   6 u8 coder (0 rANS, */
/*       1 tANS, 2 pair rANS)   7 u8 P                                       */
/*   8   u64 n    16 u32 chunk_elems   20 u32 n_chunks   24 u32 lanes=32     */
/*   28  u32 aux  32 u64 chunks_off  40 u64 plane_off  48 u64 blob_bytes     */
/*   56  version 1: u64 0; version 2: u32 groups G, u32 0                    */
/*   64  u16 freq[256]                                                       */
/* A chunk of chunk_elems values is G state groups of chunk_elems/G values   */
/* (a multiple of 256; version 1 is G = 1); group k holds elements           */
/* [k*ge, min(n, (k+1)*ge)), ge = chunk_elems/G, n_groups = ceil(n/ge).      */
/*   576 u32 group_start[n_groups+1] (16-byte units from chunks_off)         */
/*   plane_off  = rup16(576 + 4*(n_groups+1)): n bytes (sign<<7 | mantissa)  */
/*   chunks_off = plane_off + rup16(n): per group [u32 init[32]][u16 words]  */
/*                zero-padded to 16 bytes; blob_bytes = end of last record.  */
/* Element e of a group belongs to lane (e%256)/8 at step (e/256)*8 + e%8.  */
/* Coder 2 (rANS over exponent pairs): header u32 at 28 = e_lo; exponent e  */
/* maps to a = e - e_lo when 0 <= e - e_lo <= 14, else a = 15 (escape); the */
/* symbol of elements (2k, 2k+1) is a*16 + b (b = 0 for a missing second    */
/* element); lane l codes pair-steps s2 (element (s2/4)*256 + l*8 +         */
/* 2*(s2%4)); a group record is [u32 init[32]][u32 n_words][u32 n_esc][u32  */
/* 0][u32 0][u16 words][u8 escape exponents, in step/lane/a-then-b order].  */
/* ======================================================================== */
#define XC_HDR 64
#define XC_FREQ_OFF 64
#define XC_TAB_OFF 576
#define XC_LANES 32

static inline int64_t rup16(int64_t x) { return (x + 15) & ~(int64_t)15; }

int64_t bso_xc_bound(int64_t n, uint32_t chunk_elems) {
    if (chunk_elems == 0) return BSO_E_ARG;
    int64_t nc = (n + chunk_elems - 1) / chunk_elems;
    /* each symbol emits at most one u16 word per step (rANS) or at most
     * P<=12 bits (tANS); 128 B of lane state + padding per chunk */
    return rup16(XC_TAB_OFF + 4 * (nc + 1)) + nc * (128 + 16 + 32) + 2 * n + rup16(n) + 64;
}

/* deterministic frequency quantisation of the exponent histogram */
int bso_xc_quantise(const int64_t *counts, int prec, uint16_t *freqs) {
    if (prec < 8 || prec > 12) return BSO_E_ARG;
    const int64_t M = 1ll << prec;
    int nnz = 0, first = -1;
    int64_t total = 0;
    for (int s = 0; s < 256; s++) if (counts[s] > 0) { nnz++; total += counts[s]; if (first < 0) first = s; }
    for (int s = 0; s < 256; s++) freqs[s] = 0;
    if (nnz <= 1) {
        int s = first < 0 ? 0 : first;
        freqs[s] = (uint16_t)(M - 1);          /* every freq stays < M */
        freqs[(s + 1) & 255] = 1;              /* phantom symbol */
        return BSO_OK;
    }
    int64_t f[256], sum = 0;
    for (int s = 0; s < 256; s++) {
        f[s] = counts[s] > 0 ? (counts[s] * M) / total : 0;
        if (counts[s] > 0 && f[s] == 0) f[s] = 1;
        sum += f[s];
    }
    int64_t diff = M - sum;
    if (diff > 0) {
        int best = 0;
        for (int s = 1; s < 256; s++) if (f[s] > f[best]) best = s;
        f[best] += diff;
    }
    while (diff < 0) {
        int best = 0;
        for (int s = 1; s < 256; s++) if (f[s] > f[best]) best = s;
        int64_t take = f[best] - 1 < -diff ? f[best] - 1 : -diff;
        f[best] -= take;
        diff += take;
    }
    for (int s = 0; s < 256; s++) freqs[s] = (uint16_t)f[s];
    return BSO_OK;
}

/* tANS tables (FSE-style spread, Collet's step (T>>1)+(T>>3)+3):
 *   dec[i] = sym | nb<<8 | base<<12, slot_list[cum[s] + r] = r-th slot of s */
static void xc_tans_tables(const uint16_t *freq, int P, uint32_t *dec, uint16_t *slot_list, uint32_t *cum) {
    const uint32_t T = 1u << P, mask = T - 1, step = (T >> 1) + (T >> 3) + 3;
    uint8_t *spread = (uint8_t *)malloc(T);
    uint32_t c = 0, pos = 0;
    for (int s = 0; s < 256; s++) {
        cum[s] = c;
        for (uint32_t k = 0; k < freq[s]; k++) { spread[pos] = (uint8_t)s; pos = (pos + step) & mask; }
        c += freq[s];
    }
    uint32_t next[256], occ[256];
    for (int s = 0; s < 256; s++) { next[s] = freq[s]; occ[s] = 0; }
    for (uint32_t i = 0; i < T; i++) {
        uint32_t s = spread[i];
        uint32_t xs = next[s]++;
        int hb = 31 - __builtin_clz(xs);
        uint32_t nb = (uint32_t)(P - hb);
        uint32_t base = (xs << nb) - T;
        dec[i] = s | (nb << 8) | (base << 12);
        slot_list[cum[s] + occ[s]++] = (uint16_t)i;
    }
    free(spread);
}

/* growable u16 vector */
typedef struct { uint16_t *v; int64_t n, cap; } vec16;
static int v16_push(vec16 *a, uint16_t x) {
    if (a->n == a->cap) {
        int64_t nc = a->cap ? a->cap * 2 : 1024;
        uint16_t *p = (uint16_t *)realloc(a->v, sizeof(uint16_t) * (size_t)nc);
        if (!p) return -1;
        a->v = p; a->cap = nc;
    }
    a->v[a->n++] = x;
    return 0;
}

/* encode one chunk's exponents `ex[0..cn)` into `rec`, returns record bytes */
static int64_t xc_encode_chunk(const uint8_t *ex, int64_t cn, int coder, int P, const uint16_t *freq,
                               const uint32_t *cum, const uint16_t *slot_list,
                               uint8_t *rec, int64_t cap) {
    const int64_t S = ((cn + 255) / 256) * 8;
    uint32_t init[XC_LANES];
    vec16 words = {0, 0, 0};
    if (coder == 0) {
        uint64_t x[XC_LANES];
        for (int l = 0; l < XC_LANES; l++) x[l] = RANS_L;
        for (int64_t s = S - 1; s >= 0; s--) {
            int64_t g = s >> 3, j = s & 7;
            for (int l = XC_LANES - 1; l >= 0; l--) {
                int64_t e = g * 256 + l * 8 + j;
                if (e >= cn) continue;
                uint32_t sym = ex[e];
                uint64_t f = freq[sym], cf = cum[sym];
                if (x[l] >= (f << (32 - P))) { v16_push(&words, (uint16_t)(x[l] & 0xFFFF)); x[l] >>= 16; }
                x[l] = ((x[l] / f) << P) + (x[l] % f) + cf;
            }
        }
        for (int l = 0; l < XC_LANES; l++) init[l] = (uint32_t)x[l];
        /* reverse into decode order */
        for (int64_t a = 0, b = words.n - 1; a < b; a++, b--) { uint16_t t = words.v[a]; words.v[a] = words.v[b]; words.v[b] = t; }
    } else {
        const uint32_t T = 1u << P;
        /* phase 1: per-lane reverse pass producing (nb, bits) per step */
        uint8_t *nbits = (uint8_t *)malloc((size_t)(S * XC_LANES));
        uint16_t *vals = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(S * XC_LANES));
        uint32_t X[XC_LANES];
        for (int l = 0; l < XC_LANES; l++) X[l] = T;
        for (int64_t s = S - 1; s >= 0; s--) {
            int64_t g = s >> 3, j = s & 7;
            for (int l = 0; l < XC_LANES; l++) {
                int64_t e = g * 256 + l * 8 + j;
                if (e >= cn) { nbits[s * XC_LANES + l] = 0; vals[s * XC_LANES + l] = 0; continue; }
                uint32_t sym = ex[e], f = freq[sym];
                int hbx = 31 - __builtin_clz(X[l]), hbf = 31 - __builtin_clz(f);
                /* X in [T,2T): shifting by hbx-hbf lands in [2^hbf, 2^(hbf+1)),
                 * below 2f; one bit less is needed when it lands below f */
                int nb = hbx - hbf;
                if ((X[l] >> nb) < f) nb--;
                nbits[s * XC_LANES + l] = (uint8_t)nb;
                vals[s * XC_LANES + l] = (uint16_t)(X[l] & ((1u << nb) - 1));
                uint32_t xp = X[l] >> nb;
                X[l] = T + slot_list[cum[sym] + (xp - f)];
            }
        }
        /* phase 2: per-lane LSB-first bit strings */
        uint64_t acc[XC_LANES]; int accn[XC_LANES];
        vec16 lw[XC_LANES];
        for (int l = 0; l < XC_LANES; l++) { acc[l] = 0; accn[l] = 0; lw[l].v = NULL; lw[l].n = lw[l].cap = 0; }
        for (int64_t s = 0; s < S; s++)
            for (int l = 0; l < XC_LANES; l++) {
                int nb = nbits[s * XC_LANES + l];
                if (!nb) continue;
                acc[l] |= (uint64_t)vals[s * XC_LANES + l] << accn[l];
                accn[l] += nb;
                while (accn[l] >= 16) { v16_push(&lw[l], (uint16_t)acc[l]); acc[l] >>= 16; accn[l] -= 16; }
            }
        for (int l = 0; l < XC_LANES; l++) if (accn[l] > 0) v16_push(&lw[l], (uint16_t)acc[l]);
        /* phase 3: forward simulation of the decoder's refills */
        int64_t wi[XC_LANES]; int cnt[XC_LANES];
        for (int l = 0; l < XC_LANES; l++) {
            uint16_t first = lw[l].n > 0 ? lw[l].v[0] : 0;
            init[l] = (X[l] - T) | ((uint32_t)first << 16);
            wi[l] = 1; cnt[l] = 16;
        }
        for (int64_t s = 0; s < S; s++) {
            int64_t g = s >> 3, j = s & 7;
            for (int l = 0; l < XC_LANES; l++) {
                int64_t e = g * 256 + l * 8 + j;
                if (e >= cn) continue;
                if (cnt[l] < P) {
                    uint16_t wv = wi[l] < lw[l].n ? lw[l].v[wi[l]] : 0;
                    wi[l]++;
                    v16_push(&words, wv);
                    cnt[l] += 16;
                }
                cnt[l] -= nbits[s * XC_LANES + l];
            }
        }
        for (int l = 0; l < XC_LANES; l++) free(lw[l].v);
        free(nbits); free(vals);
    }
    int64_t bytes = rup16(128 + 2 * words.n);
    if (bytes > cap) { free(words.v); return BSO_E_CAP; }
    memset(rec, 0, (size_t)bytes);
    for (int l = 0; l < XC_LANES; l++) wr32(rec + 4 * l, init[l]);
    for (int64_t k = 0; k < words.n; k++) wr16(rec + 128 + 2 * k, words.v[k]);
    free(words.v);
    return bytes;
}

/* ---- coder 2: rANS over exponent pairs ---------------------------------- */
#define XC2_SAMPLE_MIN (1ll << 20)
static int xc2_window(const int64_t *hist) {
    int best = 0;
    int64_t bm = -1;
    for (int w = 0; w + 14 < 256; w++) {
        int64_t m = 0;
        for (int k = 0; k < 15; k++) m += hist[w + k];
        if (m > bm) { bm = m; best = w; }
    }
    return best;
}

static inline uint32_t xc2_a(uint32_t e, int e_lo) {
    int d = (int)e - e_lo;
    return (d >= 0 && d <= 14) ? (uint32_t)d : 15u;
}

/* pair symbol of pair-step s2 for lane l, or -1 if inactive */
static inline int xc2_sym(const uint8_t *ex, int64_t cn, int e_lo, int64_t s2, int l, int64_t *e_out) {
    int64_t e = (s2 >> 2) * 256 + l * 8 + 2 * (s2 & 3);
    if (e >= cn) return -1;
    uint32_t a = xc2_a(ex[e], e_lo);
    uint32_t b = (e + 1 < cn) ? xc2_a(ex[e + 1], e_lo) : 0u;
    *e_out = e;
    return (int)(a * 16 + b);
}

static int64_t xc2_encode_chunk(const uint8_t *ex, int64_t cn, int e_lo, int P, const uint16_t *freq,
                                const uint32_t *cum, uint8_t *rec, int64_t cap) {
    const int64_t S2 = ((cn + 255) / 256) * 4;
    uint64_t x[XC_LANES];
    vec16 words = {0, 0, 0};
    for (int l = 0; l < XC_LANES; l++) x[l] = RANS_L;
    for (int64_t s2 = S2 - 1; s2 >= 0; s2--) {
        for (int l = XC_LANES - 1; l >= 0; l--) {
            int64_t e;
            int sym = xc2_sym(ex, cn, e_lo, s2, l, &e);
            if (sym < 0) continue;
            uint64_t f = freq[sym], cf = cum[sym];
            if (x[l] >= (f << (32 - P))) { v16_push(&words, (uint16_t)(x[l] & 0xFFFF)); x[l] >>= 16; }
            x[l] = ((x[l] / f) << P) + (x[l] % f) + cf;
        }
    }
    for (int64_t a = 0, b = words.n - 1; a < b; a++, b--) { uint16_t t = words.v[a]; words.v[a] = words.v[b]; words.v[b] = t; }
    /* escapes, forward */
    int64_t n_esc = 0;
    uint8_t *esc = (uint8_t *)malloc((size_t)(cn + 1));
    for (int64_t s2 = 0; s2 < S2; s2++)
        for (int l = 0; l < XC_LANES; l++) {
            int64_t e;
            int sym = xc2_sym(ex, cn, e_lo, s2, l, &e);
            if (sym < 0) continue;
            if ((sym >> 4) == 15) esc[n_esc++] = ex[e];
            if (e + 1 < cn && (sym & 15) == 15) esc[n_esc++] = ex[e + 1];
        }
    int64_t bytes = rup16(144 + 2 * words.n + n_esc);
    if (bytes > cap) { free(words.v); free(esc); return BSO_E_CAP; }
    memset(rec, 0, (size_t)bytes);
    for (int l = 0; l < XC_LANES; l++) wr32(rec + 4 * l, (uint32_t)x[l]);
    wr32(rec + 128, (uint32_t)words.n);
    wr32(rec + 132, (uint32_t)n_esc);
    for (int64_t k = 0; k < words.n; k++) wr16(rec + 144 + 2 * k, words.v[k]);
    memcpy(rec + 144 + 2 * words.n, esc, (size_t)n_esc);
    free(words.v);
    free(esc);
    return bytes;
}

static int xc2_decode_chunk(const uint8_t *rec, int64_t rec_bytes, int64_t cn, int e_lo, int P,
                            const uint32_t *tab /* sym | f<<16 */, const uint32_t *cumf,
                            const uint8_t *plane, uint16_t *out) {
    if (rec_bytes < 144) return BSO_E_CORRUPT;
    const int64_t n_words = rd32(rec + 128), n_esc = rd32(rec + 132);
    if (rd32(rec + 136) || rd32(rec + 140)) return BSO_E_CORRUPT;
    if (144 + 2 * n_words + n_esc > rec_bytes || rec_bytes - (144 + 2 * n_words + n_esc) >= 16) return BSO_E_CORRUPT;
    const uint8_t *wd = rec + 144, *esc = rec + 144 + 2 * n_words;
    const uint32_t M = 1u << P;
    uint32_t x[XC_LANES];
    for (int l = 0; l < XC_LANES; l++) x[l] = rd32(rec + 4 * l);
    int64_t wp = 0, ep = 0;
    const int64_t S2 = ((cn + 255) / 256) * 4;
    for (int64_t s2 = 0; s2 < S2; s2++) {
        for (int l = 0; l < XC_LANES; l++) {
            int64_t e = (s2 >> 2) * 256 + l * 8 + 2 * (s2 & 3);
            if (e >= cn) continue;
            uint32_t slot = x[l] & (M - 1);
            uint32_t t = tab[slot];
            uint32_t sym = t & 0xFFFF, f = t >> 16;
            x[l] = f * (x[l] >> P) + slot - cumf[sym];
            uint32_t a = sym >> 4, b = sym & 15;
            uint32_t ea, eb = 0;
            if (a == 15) { if (ep >= n_esc) return BSO_E_CORRUPT; ea = esc[ep++]; } else ea = (uint32_t)e_lo + a;
            if (e + 1 < cn) {
                if (b == 15) { if (ep >= n_esc) return BSO_E_CORRUPT; eb = esc[ep++]; } else eb = (uint32_t)e_lo + b;
            }
            uint8_t sm = plane[e];
            out[e] = (uint16_t)(((uint32_t)(sm & 0x80) << 8) | (ea << 7) | (sm & 0x7F));
            if (e + 1 < cn) {
                sm = plane[e + 1];
                out[e + 1] = (uint16_t)(((uint32_t)(sm & 0x80) << 8) | (eb << 7) | (sm & 0x7F));
            }
            if (x[l] < RANS_L) {
                if (wp >= n_words) return BSO_E_CORRUPT;
                x[l] = (x[l] << 16) | rd16(wd + 2 * wp++);
            }
        }
    }
    for (int l = 0; l < XC_LANES; l++) if (x[l] != RANS_L) return BSO_E_CORRUPT;
    if (wp != n_words || ep != n_esc) return BSO_E_CORRUPT;
    return BSO_OK;
}

int64_t bso_xc_encode(const uint16_t *w, int64_t n, int coder, int prec, uint32_t chunk_elems,
                      uint8_t *out, int64_t cap) {
    return bso_xc_encode_groups(w, n, coder, prec, chunk_elems, 1, out, cap);
}

/* The records of a G-group blob are those of a one-group blob with       */
/* chunk_elems / G values per chunk; only the header's chunk fields and    */
/* version differ.  Below, "chunk" is the coded unit (the group).           */
int64_t bso_xc_encode_groups(const uint16_t *w, int64_t n, int coder, int prec, uint32_t chunk_elems_hdr,
                             uint32_t groups, uint8_t *out, int64_t cap) {
    if (n == 0) return 0;
    if (groups == 0 || chunk_elems_hdr == 0 || chunk_elems_hdr % groups) return BSO_E_ARG;
    const uint32_t chunk_elems = chunk_elems_hdr / groups;   /* values per group */
    if (coder < 0 || coder > 2 || prec < 8 || prec > 12 || chunk_elems == 0 || (chunk_elems & 255))
        return BSO_E_ARG;
    int64_t nc64 = (n + chunk_elems - 1) / chunk_elems;
    if (nc64 > 0x7FFFFFFFll) return BSO_E_ARG;
    uint32_t nc = (uint32_t)nc64;
    int64_t counts[256] = {0};
    uint8_t *ex = (uint8_t *)malloc((size_t)n);
    if (!ex) return BSO_E_NOMEM;
    /* coder 2 on a tensor of at least XC2_SAMPLE_MIN values counts only the */
    /* 2048-value blocks whose index is a multiple of 8                      */
    const int sampled = coder == 2 && n >= XC2_SAMPLE_MIN;
    for (int64_t i = 0; i < n; i++) {
        ex[i] = (uint8_t)((w[i] >> 7) & 0xFF);
        if (!sampled || ((i >> 11) & 7) == 0) counts[ex[i]]++;
    }
    uint16_t freq[256];
    int e_lo = 0;
    if (coder == 2) {
        /* pair-symbol counts of the product model: window-index marginals   */
        /* c(a) of the s counted values (a = 15 outside the window), m(a) =  */
        /* max(1, c(a) * 2^16 / s) for c(a) > 0, else 1 when sampled and 0   */
        /* when not; pc(a*16+b) = m(a) * m(b), plus 1 at (a_last, 0) for odd */
        /* n (the last value's pair has the phantom b = 0)                   */
        e_lo = xc2_window(counts);
        uint64_t marg[16];
        uint64_t inside = 0, counted = 0;
        for (int s = 0; s < 256; s++) counted += (uint64_t)counts[s];
        for (int a = 0; a < 15; a++) inside += (uint64_t)counts[e_lo + a];
        for (int a = 0; a < 16; a++) {
            uint64_t ca = a < 15 ? (uint64_t)counts[e_lo + a] : counted - inside;
            uint64_t q = (ca << 16) / counted;
            marg[a] = ca ? (q ? q : 1u) : (sampled ? 1u : 0u);
        }
        int64_t pc[256];
        for (int s = 0; s < 256; s++) pc[s] = (int64_t)(marg[s >> 4] * marg[s & 15]);
        if (n & 1) pc[xc2_a(ex[n - 1], e_lo) * 16] += 1;
        bso_xc_quantise(pc, prec, freq);
    } else {
        bso_xc_quantise(counts, prec, freq);
    }
    uint32_t cum[256];
    uint32_t c = 0;
    for (int s = 0; s < 256; s++) { cum[s] = c; c += freq[s]; }
    uint16_t *slot_list = NULL;
    uint32_t *dec = NULL;
    if (coder == 1) {
        slot_list = (uint16_t *)malloc(sizeof(uint16_t) << prec);
        dec = (uint32_t *)malloc(sizeof(uint32_t) << prec);
        uint32_t cum2[256];
        xc_tans_tables(freq, prec, dec, slot_list, cum2);
    }
    int64_t plane_off = rup16(XC_TAB_OFF + 4 * ((int64_t)nc + 1));
    int64_t chunks_off = plane_off + rup16(n);
    if (chunks_off > cap) { free(ex); free(slot_list); free(dec); return BSO_E_CAP; }
    memset(out, 0, (size_t)chunks_off);
    for (int64_t i = 0; i < n; i++) out[plane_off + i] = (uint8_t)(((w[i] >> 8) & 0x80) | (w[i] & 0x7F));
    int64_t pos = chunks_off;
    int rc = 0;
    for (uint32_t k = 0; k < nc; k++) {
        wr32(out + XC_TAB_OFF + 4 * k, (uint32_t)((pos - chunks_off) / 16));
        int64_t e0 = (int64_t)k * chunk_elems;
        int64_t cn = n - e0 < chunk_elems ? n - e0 : chunk_elems;
        int64_t b = coder == 2 ? xc2_encode_chunk(ex + e0, cn, e_lo, prec, freq, cum, out + pos, cap - pos)
                               : xc_encode_chunk(ex + e0, cn, coder, prec, freq, cum, slot_list, out + pos, cap - pos);
        if (b < 0) { rc = (int)b; break; }
        pos += b;
    }
    free(ex); free(slot_list); free(dec);
    if (rc) return rc;
    wr32(out + XC_TAB_OFF + 4 * nc, (uint32_t)((pos - chunks_off) / 16));
    int64_t total = pos;
    memcpy(out, "BSXC", 4);
    wr16(out + 4, groups > 1 ? 2 : 1);
    out[6] = (uint8_t)coder;
    out[7] = (uint8_t)prec;
    wr64(out + 8, (uint64_t)n);
    wr32(out + 16, chunk_elems_hdr);
    wr32(out + 20, (uint32_t)((n + chunk_elems_hdr - 1) / chunk_elems_hdr));
    wr32(out + 24, XC_LANES);
    wr32(out + 28, (uint32_t)e_lo);
    wr64(out + 32, (uint64_t)chunks_off);
    wr64(out + 40, (uint64_t)plane_off);
    wr64(out + 48, (uint64_t)total);
    wr64(out + 56, groups > 1 ? (uint64_t)groups : 0);
    for (int s = 0; s < 256; s++) wr16(out + XC_FREQ_OFF + 2 * s, freq[s]);
    return total;
}

int bso_xc_decode(const uint8_t *blob, int64_t len, int64_t n_weights, uint16_t *out) {
    if (n_weights == 0 || len == 0) return BSO_OK;
    if (len < XC_TAB_OFF) return BSO_E_TRUNC;
    if (memcmp(blob, "BSXC", 4) != 0) return BSO_E_MAGIC;
    const uint32_t ver = rd16(blob + 4);
    if (ver != 1 && ver != 2) return BSO_E_CORRUPT;
    int coder = blob[6], P = blob[7];
    int64_t n = (int64_t)rd64(blob + 8);
    uint32_t ce_hdr = rd32(blob + 16), nc_hdr = rd32(blob + 20), lanes = rd32(blob + 24);
    int64_t chunks_off = (int64_t)rd64(blob + 32), plane_off = (int64_t)rd64(blob + 40);
    int64_t total = (int64_t)rd64(blob + 48);
    if (n != n_weights) return BSO_E_COUNT;
    const uint32_t aux = rd32(blob + 28);
    /* version 2: G groups per chunk; decode works per group ("chunk" below) */
    const uint32_t G = ver == 2 ? rd32(blob + 56) : 1u;
    if (G == 0 || (ver == 2 && rd32(blob + 60) != 0) || ce_hdr == 0 || ce_hdr % G) return BSO_E_CORRUPT;
    if ((int64_t)nc_hdr != (n + ce_hdr - 1) / ce_hdr) return BSO_E_CORRUPT;
    const uint32_t ce = ce_hdr / G;
    if (coder < 0 || coder > 2 || P < 8 || P > 12 || lanes != XC_LANES || ce == 0 || (ce & 255))
        return BSO_E_CORRUPT;
    if (coder == 2 ? aux > 241 : aux != 0) return BSO_E_CORRUPT;
    if ((n + ce - 1) / ce > 0x7FFFFFFFll) return BSO_E_CORRUPT;
    const uint32_t nc = (uint32_t)((n + ce - 1) / ce);
    if (plane_off != rup16(XC_TAB_OFF + 4 * ((int64_t)nc + 1)) || chunks_off != plane_off + rup16(n) ||
        (total & 15) || total < chunks_off)
        return BSO_E_CORRUPT;
    if (total > len) return BSO_E_TRUNC;
    const uint32_t M = 1u << P;
    uint16_t freq[256];
    uint32_t cum[256], sum = 0;
    for (int s = 0; s < 256; s++) { freq[s] = rd16(blob + XC_FREQ_OFF + 2 * s); cum[s] = sum; sum += freq[s]; }
    if (sum != M) return BSO_E_CORRUPT;
    uint32_t *tab = (uint32_t *)malloc(sizeof(uint32_t) * M);
    uint16_t *slot_list = NULL;
    if (!tab) return BSO_E_NOMEM;
    if (coder == 0) {
        for (int s = 0; s < 256; s++) {
            if (freq[s] >= M) { free(tab); return BSO_E_CORRUPT; }
            for (uint32_t j = 0; j < freq[s]; j++) tab[cum[s] + j] = (uint32_t)s | ((uint32_t)freq[s] << 8) | (j << 20);
        }
    } else if (coder == 2) {
        for (int s = 0; s < 256; s++) {
            if (freq[s] >= M) { free(tab); return BSO_E_CORRUPT; }
            for (uint32_t j = 0; j < freq[s]; j++) tab[cum[s] + j] = (uint32_t)s | ((uint32_t)freq[s] << 16);
        }
    } else {
        slot_list = (uint16_t *)malloc(sizeof(uint16_t) * M);
        uint32_t cum2[256];
        xc_tans_tables(freq, P, tab, slot_list, cum2);
    }
    const uint8_t *plane = blob + plane_off;
    int rc = 0;
    for (uint32_t k = 0; k < nc && !rc; k++) {
        int64_t a = chunks_off + 16 * (int64_t)rd32(blob + XC_TAB_OFF + 4 * k);
        int64_t b = chunks_off + 16 * (int64_t)rd32(blob + XC_TAB_OFF + 4 * (k + 1));
        if (b < a + 128 || b > total) { rc = BSO_E_CORRUPT; break; }
        const uint8_t *rec = blob + a;
        if (coder == 2) {
            int64_t e0c = (int64_t)k * ce;
            int64_t cnc = n - e0c < ce ? n - e0c : ce;
            rc = xc2_decode_chunk(rec, b - a, cnc, (int)aux, P, tab, cum, plane + e0c, out + e0c);
            continue;
        }
        const int64_t navail = (b - a - 128) / 2;
        const uint8_t *wd = rec + 128;
        int64_t e0 = (int64_t)k * ce;
        int64_t cn = n - e0 < ce ? n - e0 : ce;
        int64_t S = ((cn + 255) / 256) * 8;
        int64_t wp = 0;
        if (coder == 0) {
            uint32_t x[XC_LANES];
            for (int l = 0; l < XC_LANES; l++) x[l] = rd32(rec + 4 * l);
            for (int64_t s = 0; s < S && !rc; s++) {
                int64_t g = s >> 3, j = s & 7;
                for (int l = 0; l < XC_LANES; l++) {
                    int64_t e = g * 256 + l * 8 + j;
                    if (e >= cn) continue;
                    uint32_t t = tab[x[l] & (M - 1)];
                    uint32_t sym = t & 0xFF;
                    x[l] = ((t >> 8) & 0xFFF) * (x[l] >> P) + (t >> 20);
                    uint8_t sm = plane[e0 + e];
                    out[e0 + e] = (uint16_t)(((uint32_t)(sm & 0x80) << 8) | (sym << 7) | (sm & 0x7F));
                    if (x[l] < RANS_L) {
                        if (wp >= navail) { rc = BSO_E_CORRUPT; break; }
                        x[l] = (x[l] << 16) | rd16(wd + 2 * wp++);
                    }
                }
            }
            for (int l = 0; l < XC_LANES && !rc; l++) if (x[l] != RANS_L) rc = BSO_E_CORRUPT;
        } else {
            uint32_t st[XC_LANES], buf[XC_LANES];
            int cnt[XC_LANES];
            for (int l = 0; l < XC_LANES; l++) {
                uint32_t v = rd32(rec + 4 * l);
                st[l] = v & 0xFFFF; buf[l] = v >> 16; cnt[l] = 16;
                if (st[l] >= M) rc = BSO_E_CORRUPT;
            }
            for (int64_t s = 0; s < S && !rc; s++) {
                int64_t g = s >> 3, j = s & 7;
                for (int l = 0; l < XC_LANES; l++) {
                    int64_t e = g * 256 + l * 8 + j;
                    if (e >= cn) continue;
                    if (cnt[l] < P) {
                        if (wp >= navail) { rc = BSO_E_CORRUPT; break; }
                        buf[l] |= (uint32_t)rd16(wd + 2 * wp++) << cnt[l];
                        cnt[l] += 16;
                    }
                    uint32_t t = tab[st[l]];
                    uint32_t sym = t & 0xFF, nb = (t >> 8) & 0xF;
                    st[l] = (t >> 12) + (buf[l] & ((1u << nb) - 1));
                    buf[l] >>= nb;
                    cnt[l] -= (int)nb;
                    uint8_t sm = plane[e0 + e];
                    out[e0 + e] = (uint16_t)(((uint32_t)(sm & 0x80) << 8) | (sym << 7) | (sm & 0x7F));
                }
            }
            for (int l = 0; l < XC_LANES && !rc; l++) if (st[l] != 0) rc = BSO_E_CORRUPT;
        }
        /* every word consumed; only zero padding (< 16 B) may remain */
        if (!rc && (navail - wp) * 2 >= 16) rc = BSO_E_CORRUPT;
    }
    free(tab);
    free(slot_list);
    return rc;
}

/* ======================================================================== */
/* multi-threaded decode of many blobs (timed CPU baseline)                  */
/* ======================================================================== */
typedef int (*dec_fn)(const uint8_t *, int64_t, int64_t, uint16_t *);
typedef struct {
    const uint8_t *const *blobs; const int64_t *lens, *nw; uint16_t *const *outs;
    int count; int next; int rc; pthread_mutex_t mu; dec_fn fn;
} pool_t;

static void *pool_worker(void *arg) {
    pool_t *p = (pool_t *)arg;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        int i = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (i >= p->count) break;
        int rc = p->fn(p->blobs[i], p->lens[i], p->nw[i], p->outs[i]);
        if (rc) { pthread_mutex_lock(&p->mu); if (!p->rc) p->rc = rc; pthread_mutex_unlock(&p->mu); }
    }
    return NULL;
}

static int run_pool(dec_fn fn, const uint8_t *const *blobs, const int64_t *lens, const int64_t *nw,
                    uint16_t *const *outs, int count, int threads) {
    pool_t p;
    p.blobs = blobs; p.lens = lens; p.nw = nw; p.outs = outs; p.count = count; p.next = 0; p.rc = 0; p.fn = fn;
    pthread_mutex_init(&p.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > 1024) threads = 1024;
    pthread_t th[1024];
    int started = 0;
    for (int t = 0; t < threads; t++) if (pthread_create(&th[t], NULL, pool_worker, &p) == 0) started++; else break;
    if (!started) pool_worker(&p);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&p.mu);
    return p.rc;
}

int bso_sk_decode_many(const uint8_t *const *blobs, const int64_t *lens, const int64_t *n_weights,
                       uint16_t *const *outs, int count, int threads) {
    return run_pool(bso_sk_decode, blobs, lens, n_weights, outs, count, threads);
}

int bso_tans_decode_many(const uint8_t *const *blobs, const int64_t *lens, const int64_t *n_weights,
                         uint16_t *const *outs, int count, int threads) {
    return run_pool(bso_tans_decode, blobs, lens, n_weights, outs, count, threads);
}

int bso_xc_decode_many(const uint8_t *const *blobs, const int64_t *lens, const int64_t *n_weights,
                       uint16_t *const *outs, int count, int threads) {
    return run_pool(bso_xc_decode, blobs, lens, n_weights, outs, count, threads);
}

int bso_par_decode_many(const uint8_t *const *blobs, const int64_t *lens, const int64_t *n_weights,
                        uint16_t *const *outs, int count, int threads) {
    return run_pool(bso_par_decode, blobs, lens, n_weights, outs, count, threads);
}
