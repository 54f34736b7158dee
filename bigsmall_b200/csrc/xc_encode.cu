// xc_encode.cu -- sm_100a encoder of bf16_exp_chunked_v1 (used for KV-cache
// compression and to build containers on the device).
//
// The reference compresses KV entries on the CPU after a device->host copy
// (bigsmall/codecs/kv_cache.py:24-29, :64-69).  Here the bf16 tensor never
// leaves HBM:
//   1. xc_enc_hist_kernel    exponent histogram (per-warp shared-memory bins)
//                            and the sign|mantissa byte plane, one pass.
//      Pair coder: xc_enc_expo_hist_kernel counts exponents only, over one
//      eighth of a large tensor; the setup kernel picks the 15-exponent
//      window and derives the pair-symbol counts from that histogram, as
//      products of the two window-index marginals; the chunk encoder writes
//      the plane.  The input is then read once in full, by the chunk encoder.
//   2. xc_enc_setup_kernel   deterministic frequency quantisation (the same
//                            rule as the CPU reference encoder, one symbol per
//                            thread), blob header, per-symbol encode table.
//   3. xc_enc_chunks_kernel  one warp per chunk: the 32 interleaved rANS states
//                            run backwards over the chunk; renorm words are
//                            written from the end of a per-chunk scratch slot
//                            downwards so they land in decode order.
//      xc_enc_chunks_pair_kernel  the same over exponent pairs; the escape list
//                            is written in the same backward pass, downwards.
//      xc_enc_chunks_tans_kernel  the tANS coder: a backward pass per lane, then
//                            a forward replay of the decoder's refills.
//   4. xc_enc_scan_kernel    exclusive scan of record sizes -> chunk table and
//                            blob length.
//   5. xc_enc_compact_kernel copy every record from its scratch slot into the
//                            blob, 16 bytes per thread and pass.
// Output bytes equal the CPU reference encoder's for the same input.
#include <cstdint>

#include "common.cuh"

namespace bsg {

namespace {
constexpr int kEncWarps = 4;            // chunks (warps) per CTA: small tensors still spread over SMs
constexpr uint64_t kWsCounts = 0;       // u64[256] exponent histogram
constexpr uint64_t kWsTab = 2048;       // u32[256]: freq | cum << 16
constexpr uint64_t kWsFlags = 3072;     // u32 flags
constexpr uint64_t kWsAux = 3076;       // u32 pair coder: window base e_lo
constexpr uint64_t kWsRcp = 6144;       // uint4[256]: rANS encode-step entries (rans_enc_entry)
constexpr uint64_t kWsRec = 10240;      // u32[n_chunks] words per record, then u32[n_chunks] escapes

inline uint64_t rup(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }
inline uint64_t slot_bytes(uint32_t ce) { return rup(kXcPairRecHdr + 2ull * ce, 16); }
inline uint64_t slotlist_off(uint64_t nc) { return rup(kWsRec + 8 * nc, 256); }   // u16[4096] (tANS)
inline uint64_t slots_off(uint64_t nc) { return slotlist_off(nc) + 2 * kXcMaxTable; }
// tANS: one u32 (bits | nbits << 16) per lane and step, rup(chunk, 256) per chunk
inline uint64_t tans_scratch_off(uint64_t nc, uint32_t ce) { return slots_off(nc) + nc * slot_bytes(ce); }
}  // namespace

uint64_t xc_encode_workspace(uint64_t n, uint32_t ce, int coder) {
    uint64_t nc = (n + ce - 1) / ce;
    uint64_t b = slots_off(nc) + nc * slot_bytes(ce);
    if (coder == BS_CODER_TANS) b += nc * 4ull * rup(ce, 256);
    return b;
}

uint64_t xc_encode_bound(uint64_t n, uint32_t ce) {
    uint64_t nc = (n + ce - 1) / ce;
    uint64_t plane_off = rup(kXcTabOff + 4 * (nc + 1), 16);
    return plane_off + rup(n, 16) + nc * slot_bytes(ce);
}

__device__ __forceinline__ uint32_t lanemask_gt_e() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_gt;" : "=r"(m));
    return m;
}

// one streaming 16-byte read of the input (read once per pass: no L1
// allocation, 256-byte L2 fills)
__device__ __forceinline__ uint4 ld_stream16(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 1. histogram + plane ------------------------------------------------------
__global__ void __launch_bounds__(256) xc_enc_hist_kernel(const uint16_t *__restrict__ in, uint64_t n,
                                                          unsigned long long *counts,
                                                          uint8_t *__restrict__ plane) {
    __shared__ uint32_t h[8][256];
    const uint32_t w = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 8 * 256; i += 256) (&h[0][0])[i] = 0;
    __syncthreads();
    const uint64_t n8 = n / 8;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t q = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; q < n8; q += stride) {
        uint4 v = ld_stream16(reinterpret_cast<const uint4 *>(in) + q);
        uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t pl[2] = {0, 0};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            uint32_t lo = wv[k] & 0xFFFF, hi = wv[k] >> 16;
            atomicAdd(&h[w][(lo >> 7) & 0xFF], 1u);
            atomicAdd(&h[w][(hi >> 7) & 0xFF], 1u);
            uint32_t b0 = ((lo >> 8) & 0x80) | (lo & 0x7F), b1 = ((hi >> 8) & 0x80) | (hi & 0x7F);
            pl[k >> 1] |= (b0 | (b1 << 8)) << ((k & 1) * 16);
        }
        reinterpret_cast<uint2 *>(plane)[q] = make_uint2(pl[0], pl[1]);
    }
    if (blockIdx.x == 0) {
        for (uint64_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) {
            uint32_t v = in[i];
            atomicAdd(&h[w][(v >> 7) & 0xFF], 1u);
            plane[i] = static_cast<uint8_t>(((v >> 8) & 0x80) | (v & 0x7F));
        }
    }
    __syncthreads();
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) s += h[k][threadIdx.x];
    if (s) atomicAdd(&counts[threadIdx.x], static_cast<unsigned long long>(s));
}

// 1b. pair coder: exponent histogram only (its chunk encoder writes the plane).
// A tensor of at least kSampleMin values is sampled: the values of the
// 2048-value blocks whose index is a multiple of 8, one eighth of the input
// (2048 values are 256 16-byte vectors, so vector q is sampled when
// q mod 2048 < 256).  The pair coder's escapes keep its alphabet closed (16
// window indices), so a sampled histogram can never leave a coded symbol
// without a frequency once every window index gets one (the window kernel).
constexpr uint64_t kSampleMin = 1ull << 20;

__host__ __device__ inline uint64_t sampled_vectors(uint64_t n8) {
    return (n8 >> 11) * 256 + (((n8 & 2047) < 256) ? (n8 & 2047) : 256);
}

__global__ void __launch_bounds__(256) xc_enc_expo_hist_kernel(const uint16_t *__restrict__ in, uint64_t n,
                                                               unsigned long long *counts) {
    __shared__ uint32_t h[8][256];
    const uint32_t w = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 8 * 256; i += 256) (&h[0][0])[i] = 0;
    __syncthreads();
    const bool sample = n >= kSampleMin;
    const uint64_t n8 = n / 8;
    const uint64_t nv = sample ? sampled_vectors(n8) : n8;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t k = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; k < nv; k += stride) {
        const uint64_t q = sample ? ((k >> 8) << 11) | (k & 255) : k;
        const uint4 v = ld_stream16(reinterpret_cast<const uint4 *>(in) + q);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            atomicAdd(&h[w][(wv[j] >> 7) & 0xFF], 1u);
            atomicAdd(&h[w][(wv[j] >> 23) & 0xFF], 1u);
        }
    }
    if (blockIdx.x == 0) {
        for (uint64_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x)
            if (!sample || ((i >> 11) & 7) == 0) atomicAdd(&h[w][(in[i] >> 7) & 0xFF], 1u);
    }
    __syncthreads();
    uint32_t t = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) t += h[k][threadIdx.x];
    if (t) atomicAdd(&counts[threadIdx.x], static_cast<unsigned long long>(t));
}

// 2a. pair coder: exponent window and pair-symbol counts (in the setup block) -
__device__ __forceinline__ uint32_t pair_a(uint32_t v, uint32_t e_lo) {
    const uint32_t d = ((v >> 7) & 0xFF) - e_lo;   // wraps to a large value below e_lo
    return min(d, 15u);
}

// The 15-wide exponent window holding the most values (lowest base on ties):
// thread w sums window w, then a max reduction keeps the lowest w among equals.
// Then the pair-symbol counts the frequencies are quantised from (a product
// model: a pair codes two neighbouring values, whose exponents are close to
// independent, so this costs about 0.001-0.007 bits per value against the
// pairs' own histogram and saves a pass over the input):
//   s     values the histogram counted (n, or the sample of xc_enc_expo_hist_kernel),
//   c(a)  counted values with window index a (a = 15: outside the window),
//   m(a)  = max(1, c(a) * 2^16 / s) if c(a) > 0; else 1 for a sampled
//         histogram (the rest of the tensor may hold such values), 0 otherwise,
//   pc(a*16 + b) = m(a) * m(b), plus 1 at (a of the last value, 0) when n is
//   odd (that value's pair has the phantom b = 0, so its symbol needs f > 0).
// Run by all 256 threads of the setup block; returns pc(threadIdx.x) and
// stores e_lo at *aux.
__device__ unsigned long long pair_counts_block(const unsigned long long *counts,
                                                const uint16_t *__restrict__ in, uint64_t n, uint32_t *aux) {
    __shared__ unsigned long long c[256];
    __shared__ unsigned long long s_m[8];
    __shared__ uint32_t s_w[8];
    __shared__ unsigned long long s_marg[16];
    __shared__ uint32_t s_elo;
    const uint32_t t = threadIdx.x, lane = t & 31;
    c[t] = counts[t];
    __syncthreads();
    unsigned long long m = 0;
    uint32_t w = 0xFFFFu;                         // not a window: loses every comparison
    if (t + 14 < 256) {
        for (int k = 0; k < 15; k++) m += c[t + k];
        w = t;
    }
    auto better = [](unsigned long long m1, uint32_t w1, unsigned long long m0, uint32_t w0) {
        return m1 > m0 || (m1 == m0 && w1 < w0);
    };
    for (int off = 16; off; off >>= 1) {
        const unsigned long long om = __shfl_down_sync(kFull, m, off);
        const uint32_t ow = __shfl_down_sync(kFull, w, off);
        if (better(om, ow, m, w)) { m = om; w = ow; }
    }
    if (lane == 0) { s_m[t >> 5] = m; s_w[t >> 5] = w; }
    __syncthreads();
    if (t == 0) {
        for (int k = 1; k < 8; k++)
            if (better(s_m[k], s_w[k], m, w)) { m = s_m[k]; w = s_w[k]; }
        *aux = w;
        s_elo = w;
    }
    __syncthreads();
    const uint32_t e_lo = s_elo;
    if (t < 16) {
        unsigned long long counted = 0, inside = 0;
        for (int k = 0; k < 256; k++) counted += c[k];
        for (int k = 0; k < 15; k++) inside += c[e_lo + k];
        const unsigned long long ca = t < 15 ? c[e_lo + t] : counted - inside;
        const unsigned long long q = (ca << 16) / counted;
        s_marg[t] = ca ? (q ? q : 1ull) : (n >= kSampleMin ? 1ull : 0ull);
    }
    __syncthreads();
    unsigned long long pc = s_marg[t >> 4] * s_marg[t & 15];
    if ((n & 1) && t == pair_a(in[n - 1], e_lo) * 16) pc += 1;
    return pc;
}

// 2. quantise + header -----------------------------------------------------
// Same rule as the CPU reference encoder of the format: f = max(1, c*M/total)
// for present symbols; a positive remainder goes to the most frequent symbol
// (lowest index on ties); an excess is taken from the most frequent symbols,
// never below 1; a single present symbol gets M-1 plus a phantom neighbour.
// `ce` / `nc` are the values per state group and the group count (the coded
// units); the header names chunks of ce * groups values.
__global__ void __launch_bounds__(256) xc_enc_setup_kernel(const unsigned long long *counts,
                                                           const uint16_t *__restrict__ in, uint64_t n,
                                                           int coder, int prec, uint32_t ce, uint32_t nc,
                                                           uint32_t groups, uint8_t *out, uint32_t *enc_tab,
                                                           uint16_t *slot_list, uint32_t *aux) {
    __shared__ int64_t f[256];
    __shared__ uint32_t s_cum[256];
    __shared__ uint8_t s_spread[kXcMaxTable];
    __shared__ uint32_t s_occ[256];
    __shared__ unsigned long long s_red64[8];
    __shared__ uint32_t s_red[8];
    const int tid = threadIdx.x;
    const uint32_t lane = tid & 31, warp = tid >> 5;
    const int64_t M = 1ll << prec;
    // One symbol per thread; the sequential steps of the rule (the remainder
    // and excess go to the most frequent symbol, lowest index on ties) become
    // block reductions over (freq << 8 | 255 - symbol).
    auto block_max = [&](uint32_t k) -> uint32_t {
        k = __reduce_max_sync(0xFFFFFFFFu, k);
        __syncthreads();   // the previous reduction's readers are done
        if (lane == 0) s_red[warp] = k;
        __syncthreads();
        uint32_t r = s_red[0];
#pragma unroll
        for (int w = 1; w < 8; w++) r = max(r, s_red[w]);
        return r;
    };
    auto block_add = [&](uint32_t k) -> uint32_t {
        k = __reduce_add_sync(0xFFFFFFFFu, k);
        __syncthreads();
        if (lane == 0) s_red[warp] = k;
        __syncthreads();
        uint32_t r = 0;
#pragma unroll
        for (int w = 0; w < 8; w++) r += s_red[w];
        return r;
    };
    // the pair coder quantises its pair-symbol counts (window and product
    // model above); the others the exponent histogram itself
    const unsigned long long c = coder == BS_CODER_RANS_PAIR ? pair_counts_block(counts, in, n, aux) : counts[tid];
    unsigned long long tot = c;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, d);
    if (lane == 0) s_red64[warp] = tot;
    const int nnz = __syncthreads_count(c != 0);
    unsigned long long total = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) total += s_red64[w];
    int64_t v;
    if (nnz <= 1) {
        // the present symbol (0 if none) gets M-1, its successor a phantom 1
        const uint32_t first = 255u - (block_max(c ? 255u - tid : 0u) & 255u);
        const uint32_t s = nnz ? first : 0u;
        v = tid == static_cast<int>(s) ? M - 1 : (tid == static_cast<int>((s + 1) & 255) ? 1 : 0);
        f[tid] = v;
    } else {
        // c < 2^51 for any tensor that fits in memory, so c*M fits in 64 bits
        v = c ? static_cast<int64_t>((c * static_cast<unsigned long long>(M)) / total) : 0;
        if (c && v == 0) v = 1;
        f[tid] = v;
        int64_t diff = M - static_cast<int64_t>(block_add(static_cast<uint32_t>(v)));
        while (diff != 0) {   // uniform: every thread sees the same diff
            const uint32_t best = 255u - (block_max((static_cast<uint32_t>(f[tid]) << 8) | (255u - tid)) & 255u);
            if (diff > 0) {
                if (tid == static_cast<int>(best)) f[tid] += diff;
                diff = 0;
            } else {
                const int64_t fb = f[best];
                const int64_t take = fb - 1 < -diff ? fb - 1 : -diff;
                __syncthreads();   // everyone has read f[best]
                if (tid == static_cast<int>(best)) f[tid] -= take;
                diff += take;
            }
            __syncthreads();
        }
    }
    __syncthreads();
    {
        // exclusive prefix sum of the frequencies
        const uint32_t fv = static_cast<uint32_t>(f[tid]);
        uint32_t incl = fv;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t o = __shfl_up_sync(0xFFFFFFFFu, incl, d);
            if (lane >= static_cast<uint32_t>(d)) incl += o;
        }
        __syncthreads();
        if (lane == 31) s_red[warp] = incl;
        __syncthreads();
        uint32_t base = 0;
        for (uint32_t w = 0; w < warp; w++) base += s_red[w];
        s_cum[tid] = base + incl - fv;
    }
    __syncthreads();
    // header
    const uint64_t plane_off = (kXcTabOff + 4ull * (nc + 1ull) + 15) & ~15ull;
    const uint64_t chunks_off = plane_off + ((n + 15) & ~15ull);
    if (tid == 0) {
        uint32_t *h32 = reinterpret_cast<uint32_t *>(out);
        uint64_t *h64 = reinterpret_cast<uint64_t *>(out);
        const uint64_t ce_hdr = static_cast<uint64_t>(ce) * groups;
        h32[0] = kXcMagic;
        h32[1] = (groups > 1 ? 2u : 1u) | (static_cast<uint32_t>(coder) << 16) | (static_cast<uint32_t>(prec) << 24);
        h64[1] = n;
        h32[4] = static_cast<uint32_t>(ce_hdr);
        h32[5] = static_cast<uint32_t>((n + ce_hdr - 1) / ce_hdr);
        h32[6] = kXcLanes;
        h32[7] = coder == BS_CODER_RANS_PAIR ? *aux : 0u;
        h64[4] = chunks_off;
        h64[5] = plane_off;
        h64[7] = groups > 1 ? groups : 0u;   // version 2: u32 groups, u32 0
    }
    reinterpret_cast<uint16_t *>(out + kXcFreqOff)[tid] = static_cast<uint16_t>(f[tid]);
    // zero the two alignment pads
    const uint64_t tab_end = kXcTabOff + 4ull * (nc + 1ull);
    if (tab_end + tid < plane_off) out[tab_end + tid] = 0;
    if (plane_off + n + tid < chunks_off) out[plane_off + n + tid] = 0;
    enc_tab[tid] = static_cast<uint32_t>(f[tid]) | (s_cum[tid] << 16);
    // per-symbol encode-step entries of the rANS encoders (renorm threshold,
    // divide-by-frequency as a multiplication, cum and M - f)
    reinterpret_cast<uint4 *>(enc_tab + (kWsRcp - kWsTab) / 4)[tid] =
        rans_enc_entry(static_cast<uint32_t>(f[tid]), s_cum[tid], static_cast<uint32_t>(prec));
    if (coder != BS_CODER_TANS) return;
    // tANS: spread the symbols over the 2^P states with Collet's step (the k-th
    // placement in symbol order lands on (k * step) mod M), then list each
    // symbol's states in increasing order (the encoder's next-state table)
    const uint32_t Mu = static_cast<uint32_t>(M), step = (Mu >> 1) + (Mu >> 3) + 3;
    for (uint32_t k = tid; k < Mu; k += blockDim.x) {
        int lo = 0, hi = 255;   // largest symbol with cum <= k (it has f > 0)
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_cum[mid] <= k) lo = mid; else hi = mid - 1;
        }
        s_spread[(k * step) & (Mu - 1)] = static_cast<uint8_t>(lo);
    }
    s_occ[tid] = 0;
    __syncthreads();
    if (tid < 32) {
        uint32_t lt;
        asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
        for (uint32_t i0 = 0; i0 < Mu; i0 += 32) {
            const uint32_t i = i0 + tid;
            const uint32_t sym = s_spread[i];
            const uint32_t grp = __match_any_sync(0xFFFFFFFFu, sym);
            slot_list[s_cum[sym] + s_occ[sym] + __popc(grp & lt)] = static_cast<uint16_t>(i);
            __syncwarp();
            if ((grp & lt) == 0) s_occ[sym] += __popc(grp);
            __syncwarp();
        }
    }
}

// 3c. per-chunk reverse rANS over exponent pairs, with the escape list -------
__global__ void __launch_bounds__(kEncWarps * 32) xc_enc_chunks_pair_kernel(
    const uint16_t *__restrict__ in, uint64_t n, uint32_t ce, uint32_t nc,
    const uint4 *__restrict__ rcp_tab, const uint32_t *aux, uint8_t *__restrict__ slots, uint64_t slot_b,
    uint32_t *__restrict__ rec_words, uint32_t *__restrict__ rec_esc, uint8_t *__restrict__ plane) {
    __shared__ uint4 s_tab[256];
    for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) s_tab[i] = rcp_tab[i];
    __syncthreads();
    const uint32_t e_lo = *aux;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t c = blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (c >= nc) return;
    const uint64_t e0 = static_cast<uint64_t>(c) * ce;
    const uint32_t cn = (n - e0) < ce ? static_cast<uint32_t>(n - e0) : ce;
    const uint16_t *src = in + e0;
    uint8_t *slot = slots + static_cast<uint64_t>(c) * slot_b;
    uint16_t *wend = reinterpret_cast<uint16_t *>(slot + slot_b);
    const uint32_t gt = lanemask_gt_e();
    uint32_t lt;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
    uint32_t x = kRansL, cur = 0;
    const uint32_t G = cn >> 8, rem = cn & 255;
    // Escapes are written during the backward pass, downwards from eend: a
    // pair-step's escapes (lanes in order, first value then second) go just
    // below those of the later steps, so the list ends up in forward order in
    // [eend - n_esc, eend).  At most one renorm word per lane and pair-step
    // keeps the words (<= ce bytes, downwards from the slot end) above eend.
    uint8_t *eend = slot + kXcPairRecHdr + ce;
    uint32_t ecur = 0;

    // x <- (x / f) << P | (x mod f) + cum  ==  x + cum + (x / f) (M - f)
    uint16_t *wtop = wend - 1;   // the next word goes to wtop[-cur - (emitting lanes below)]
    // one pair-step: w holds the lane's two values (first in the low half)
    // `chk` false: the caller has seen that no lane's values escape the window
    auto enc = [&](uint32_t w, bool act, bool has_b, bool chk = true) {
        // window index: exponent - e_lo, 15 (escape) outside the window
        const uint32_t da = ((w >> 7) & 0xFF) - e_lo, db = ((w >> 23) & 0xFF) - e_lo;
        const bool ea = act && da > 14, eb = has_b && db > 14;
        const uint32_t a = act ? min(da, 15u) : 0u, b = has_b ? min(db, 15u) : 0u;
        if (chk && __ballot_sync(kFull, ea || eb)) {   // rare: only then the per-value ballots
            const uint32_t ba = __ballot_sync(kFull, ea), bb = __ballot_sync(kFull, eb);
            const int64_t k = static_cast<int64_t>(ecur) + __popc(ba) + __popc(bb);
            const int64_t pa = static_cast<int64_t>(__popc(ba & lt) + __popc(bb & lt)) - k;
            if (ea) eend[pa] = static_cast<uint8_t>((w >> 7) & 0xFF);
            if (eb) eend[pa + (ea ? 1 : 0)] = static_cast<uint8_t>((w >> 23) & 0xFF);
            ecur = static_cast<uint32_t>(k);
        }
        const uint4 t = s_tab[a * 16 + b];
        const bool emit = act && x >= t.z;   // t.z = f << (32 - P)
        const uint32_t m = __ballot_sync(kFull, emit);
        if (emit) wtop[-static_cast<int32_t>(cur + __popc(m & gt))] = static_cast<uint16_t>(x);
        x = emit ? x >> 16 : x;
        cur += __popc(m);
        if (act) x = rans_enc_update(x, t);
    };
    uint8_t *pl = plane + e0;
    if (rem) {
        const uint32_t eb = G * 256 + lane * 8;
        for (int jj = 3; jj >= 0; jj--) {
            const uint32_t e = lane * 8 + 2 * jj;
            const bool act = e < rem, has_b = e + 1 < rem;
            const uint32_t va = act ? static_cast<uint32_t>(src[eb + 2 * jj]) : 0u;
            const uint32_t vb = has_b ? static_cast<uint32_t>(src[eb + 2 * jj + 1]) : 0u;
            if (act) pl[eb + 2 * jj] = static_cast<uint8_t>(((va >> 8) & 0x80) | (va & 0x7F));
            if (has_b) pl[eb + 2 * jj + 1] = static_cast<uint8_t>(((vb >> 8) & 0x80) | (vb & 0x7F));
            enc(va | (vb << 16), act, has_b);
        }
    }
    // sign|mantissa bytes of a word's two values at bits 0-7 and 16-23
    auto sm2 = [](uint32_t w) { return (w & 0x007F007Fu) | ((w >> 8) & 0x00800080u); };
    // groups run backwards; the next two groups' values are in flight
    auto grp = [&](int g) { return reinterpret_cast<const uint4 *>(src + g * 256 + lane * 8)[0]; };
    uint4 n1 = make_uint4(0, 0, 0, 0), n2 = n1;
    if (G > 0) n1 = grp(static_cast<int>(G) - 1);
    if (G > 1) n2 = grp(static_cast<int>(G) - 2);
    for (int g = static_cast<int>(G) - 1; g >= 0; g--) {
        const uint4 v = n1;
        n1 = n2;
        if (g >= 2) n2 = grp(g - 2);
        reinterpret_cast<uint2 *>(pl + g * 256 + lane * 8)[0] =
            make_uint2(__byte_perm(sm2(v.x), sm2(v.y), 0x6420), __byte_perm(sm2(v.z), sm2(v.w), 0x6420));
        // one vote per group on escapes (window index > 14 among the lane's 8
        // values); the four pair-steps vote again only when one is there
        auto dmax = [&](uint32_t w) { return max(((w >> 7) & 0xFF) - e_lo, ((w >> 23) & 0xFF) - e_lo); };
        if (__any_sync(kFull, max(max(dmax(v.x), dmax(v.y)), max(dmax(v.z), dmax(v.w))) > 14)) {
            enc(v.w, true, true);
            enc(v.z, true, true);
            enc(v.y, true, true);
            enc(v.x, true, true);
        } else {
            enc(v.w, true, true, false);
            enc(v.z, true, true, false);
            enc(v.y, true, true, false);
            enc(v.x, true, true, false);
        }
    }
    reinterpret_cast<uint32_t *>(slot)[lane] = x;
    if (lane == 0) {
        rec_words[c] = cur;
        rec_esc[c] = ecur;
    }
}

// 3. per-chunk reverse rANS ---------------------------------------------------
__global__ void __launch_bounds__(kEncWarps * 32) xc_enc_chunks_kernel(
    const uint16_t *__restrict__ in, uint64_t n, uint32_t ce, uint32_t nc,
    const uint4 *__restrict__ rcp_tab, uint8_t *__restrict__ slots, uint64_t slot_b,
    uint32_t *__restrict__ rec_words) {
    __shared__ uint4 s_tab[256];
    for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) s_tab[i] = rcp_tab[i];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t c = blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (c >= nc) return;
    const uint64_t e0 = static_cast<uint64_t>(c) * ce;
    const uint32_t cn = (n - e0) < ce ? static_cast<uint32_t>(n - e0) : ce;
    const uint16_t *src = in + e0;
    uint8_t *slot = slots + static_cast<uint64_t>(c) * slot_b;
    uint16_t *wend = reinterpret_cast<uint16_t *>(slot + slot_b);   // words grow downwards
    const uint32_t gt = lanemask_gt_e();
    uint32_t x = kRansL;
    uint32_t cur = 0;
    const uint32_t G = cn >> 8, rem = cn & 255;

    // x <- (x / f) << P | (x mod f) + cum  ==  x + cum + (x / f) (M - f)
    auto enc = [&](uint32_t v, bool active) {
        const uint32_t sym = (v >> 7) & 0xFF;
        const uint4 t = s_tab[sym];
        const bool emit = active && x >= t.z;   // t.z = f << (32 - P)
        const uint32_t m = __ballot_sync(kFull, emit);
        if (emit) {
            wend[-1 - static_cast<int64_t>(cur + __popc(m & gt))] = static_cast<uint16_t>(x & 0xFFFF);
            x >>= 16;
        }
        cur += __popc(m);
        if (active) x = rans_enc_update(x, t);
    };

    if (rem) {
        const uint32_t eb = G * 256 + lane * 8;
        uint32_t v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = (lane * 8 + j < rem) ? src[eb + j] : 0u;
#pragma unroll
        for (int j = 7; j >= 0; j--) enc(v[j], lane * 8 + j < rem);
    }
    // groups run backwards; the next two groups' values are in flight
    auto grp = [&](int g) { return reinterpret_cast<const uint4 *>(src + g * 256 + lane * 8)[0]; };
    uint4 n1 = make_uint4(0, 0, 0, 0), n2 = n1;
    if (G > 0) n1 = grp(static_cast<int>(G) - 1);
    if (G > 1) n2 = grp(static_cast<int>(G) - 2);
    for (int g = static_cast<int>(G) - 1; g >= 0; g--) {
        const uint4 v = n1;
        n1 = n2;
        if (g >= 2) n2 = grp(g - 2);
        enc(v.w >> 16, true);
        enc(v.w & 0xFFFF, true);
        enc(v.z >> 16, true);
        enc(v.z & 0xFFFF, true);
        enc(v.y >> 16, true);
        enc(v.y & 0xFFFF, true);
        enc(v.x >> 16, true);
        enc(v.x & 0xFFFF, true);
    }
    reinterpret_cast<uint32_t *>(slot)[lane] = x;
    if (lane == 0) rec_words[c] = cur;
}

// 3b. per-chunk tANS ------------------------------------------------------------
// Phase 1 runs each lane's tANS state backwards over its symbols and records
// (bits, nbits) per step; phase 2 replays the decoder forwards: before a step,
// lanes holding fewer than P bits take their next 16-bit word of their own
// LSB-first bit string, in lane order, into the shared word stream.
__global__ void __launch_bounds__(kEncWarps * 32) xc_enc_chunks_tans_kernel(
    const uint16_t *__restrict__ in, uint64_t n, uint32_t ce, uint32_t nc, int prec,
    const uint32_t *__restrict__ enc_tab, const uint16_t *__restrict__ slot_list, uint8_t *__restrict__ slots,
    uint64_t slot_b, uint32_t *__restrict__ scratch, uint32_t *__restrict__ rec_words) {
    __shared__ uint32_t s_tab[256];
    __shared__ uint16_t s_sl[kXcMaxTable];
    const uint32_t M = 1u << prec;
    for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) s_tab[i] = enc_tab[i];
    for (uint32_t i = threadIdx.x; i < M; i += blockDim.x) s_sl[i] = slot_list[i];
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t c = blockIdx.x * kEncWarps + (threadIdx.x >> 5);
    if (c >= nc) return;
    const uint32_t P = static_cast<uint32_t>(prec);
    const uint64_t e0 = static_cast<uint64_t>(c) * ce;
    const uint32_t cn = (n - e0) < ce ? static_cast<uint32_t>(n - e0) : ce;
    const uint16_t *src = in + e0;
    uint8_t *slot = slots + static_cast<uint64_t>(c) * slot_b;
    uint32_t *sc = scratch + static_cast<uint64_t>(c) * ((ce + 255) & ~255u);
    const uint32_t G = cn >> 8, rem = cn & 255;
    const uint32_t S = (G + (rem ? 1u : 0u)) * 8;

    uint32_t X = M;
    auto enc1 = [&](uint32_t s, uint32_t v, bool active) {
        uint32_t r = 0;
        if (active) {
            const uint32_t t = s_tab[(v >> 7) & 0xFF];
            const uint32_t f = t & 0xFFFF, cf = t >> 16;
            int nb = (31 - __clz(X)) - (31 - __clz(f));
            if ((X >> nb) < f) nb--;
            const uint32_t bits = X & ((1u << nb) - 1);
            X = M + s_sl[cf + (X >> nb) - f];
            r = bits | (static_cast<uint32_t>(nb) << 16);
        }
        sc[s * 32 + lane] = r;
    };
    if (rem) {
        const uint32_t eb = G * 256 + lane * 8;
        for (int j = 7; j >= 0; j--) {
            const bool act = lane * 8 + j < rem;
            enc1(G * 8 + j, act ? src[eb + j] : 0u, act);
        }
    }
    for (int g = static_cast<int>(G) - 1; g >= 0; g--) {
        const uint4 v = reinterpret_cast<const uint4 *>(src + g * 256 + lane * 8)[0];
        enc1(g * 8 + 7, v.w >> 16, true);
        enc1(g * 8 + 6, v.w & 0xFFFF, true);
        enc1(g * 8 + 5, v.z >> 16, true);
        enc1(g * 8 + 4, v.z & 0xFFFF, true);
        enc1(g * 8 + 3, v.y >> 16, true);
        enc1(g * 8 + 2, v.y & 0xFFFF, true);
        enc1(g * 8 + 1, v.x >> 16, true);
        enc1(g * 8 + 0, v.x & 0xFFFF, true);
    }
    // phase 2
    uint64_t acc = 0;
    uint32_t accn = 0, p = 0;
    auto pull16 = [&]() -> uint32_t {
        while (accn < 16 && p < S) {
            const uint32_t r = sc[p * 32 + lane];
            acc |= static_cast<uint64_t>(r & 0xFFFF) << accn;
            accn += r >> 16;
            p++;
        }
        const uint32_t w = static_cast<uint32_t>(acc & 0xFFFF);
        acc >>= 16;
        accn = accn > 16 ? accn - 16 : 0;
        return w;
    };
    const uint32_t first = pull16();
    const uint32_t init = (X - M) | (first << 16);
    uint16_t *wout = reinterpret_cast<uint16_t *>(slot + 128);
    uint32_t lt;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
    uint32_t cnt = 16, base = 0;
    for (uint32_t s = 0; s < S; s++) {
        const bool active = (s >> 3) < G || (lane * 8 + (s & 7)) < rem;
        const bool need = active && cnt < P;
        const uint32_t m = __ballot_sync(kFull, need);
        if (need) {
            wout[base + __popc(m & lt)] = static_cast<uint16_t>(pull16());
            cnt += 16;
        }
        base += __popc(m);
        if (active) cnt -= sc[s * 32 + lane] >> 16;
    }
    reinterpret_cast<uint32_t *>(slot)[lane] = init;
    if (lane == 0) rec_words[c] = base;
}

// 4. record offsets -----------------------------------------------------------
__device__ __forceinline__ uint64_t rec16(const uint32_t *rec_words, const uint32_t *rec_esc, uint32_t c, int coder) {
    return coder == BS_CODER_RANS_PAIR ? (kXcPairRecHdr + 2ull * rec_words[c] + rec_esc[c] + 15u) >> 4
                                       : (128ull + 2ull * rec_words[c] + 15u) >> 4;
}

__global__ void __launch_bounds__(1024) xc_enc_scan_kernel(const uint32_t *__restrict__ rec_words,
                                                           const uint32_t *__restrict__ rec_esc, int coder, uint32_t nc,
                                                           uint8_t *out, uint64_t chunks_off, uint64_t out_cap,
                                                           unsigned long long *out_len, uint32_t *flags) {
    __shared__ uint64_t s_warp[32];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t per = (nc + 1023) / 1024;
    const uint32_t lo = tid * per, hi = min(nc, lo + per);
    uint64_t sum = 0;
    for (uint32_t c = lo; c < hi; c++) sum += rec16(rec_words, rec_esc, c, coder);
    // block-wide inclusive scan of the per-thread sums: within each warp by
    // shuffles, then over the 32 warp totals by the first warp
    uint64_t inc = sum;
#pragma unroll
    for (uint32_t d = 1; d < 32; d <<= 1) {
        const uint64_t v = __shfl_up_sync(kFull, inc, d);
        if (lane >= d) inc += v;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        uint64_t t = s_warp[lane];
#pragma unroll
        for (uint32_t d = 1; d < 32; d <<= 1) {
            const uint64_t v = __shfl_up_sync(kFull, t, d);
            if (lane >= d) t += v;
        }
        s_warp[lane] = t;
    }
    __syncthreads();
    uint64_t run = (warp ? s_warp[warp - 1] : 0ull) + inc - sum;   // exclusive
    uint32_t *tab = reinterpret_cast<uint32_t *>(out + kXcTabOff);
    for (uint32_t c = lo; c < hi; c++) {
        tab[c] = static_cast<uint32_t>(run);
        run += rec16(rec_words, rec_esc, c, coder);
    }
    if (tid == 1023) {
        const uint64_t total16 = s_warp[31];
        tab[nc] = static_cast<uint32_t>(total16);
        const uint64_t total = chunks_off + 16 * total16;
        if (total > out_cap) {
            *flags = 1;
            *out_len = 0;
        } else {
            *flags = 0;
            reinterpret_cast<uint64_t *>(out)[6] = total;
            *out_len = total;
        }
    }
}

// 5. compaction -----------------------------------------------------------------
// Four bytes from any address: one aligned load, or two and a funnel shift.
// Only the aligned words holding the four bytes are read.
__device__ __forceinline__ uint32_t ld_u32_any(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~static_cast<uintptr_t>(3));
    const uint32_t k = static_cast<uint32_t>(a & 3);
    if (k == 0) return base[0];
    return __funnelshift_r(base[0], base[1], 8 * k);
}

// 16 bytes from any address: the two aligned 16-byte blocks holding them,
// funnel-shifted (nothing outside those blocks is read).  The misalignment is
// the same for every piece of a record's region, so the switch is uniform.
__device__ __forceinline__ uint4 ld_u128_any(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint4 *b = reinterpret_cast<const uint4 *>(a & ~static_cast<uintptr_t>(15));
    const uint32_t k = static_cast<uint32_t>(a & 15);
    if (k == 0) return b[0];
    const uint4 lo = b[0], hi = b[1];
    const uint32_t s = 8 * (k & 3);
    auto f = [s](uint32_t x, uint32_t y) { return __funnelshift_r(x, y, s); };
    switch (k >> 2) {
        case 0: return make_uint4(f(lo.x, lo.y), f(lo.y, lo.z), f(lo.z, lo.w), f(lo.w, hi.x));
        case 1: return make_uint4(f(lo.y, lo.z), f(lo.z, lo.w), f(lo.w, hi.x), f(hi.x, hi.y));
        case 2: return make_uint4(f(lo.z, lo.w), f(lo.w, hi.x), f(hi.x, hi.y), f(hi.y, hi.z));
        default: return make_uint4(f(lo.w, hi.x), f(hi.x, hi.y), f(hi.y, hi.z), f(hi.z, hi.w));
    }
}

__global__ void __launch_bounds__(256) xc_enc_compact_kernel(const uint8_t *__restrict__ slots, uint64_t slot_b,
                                                             const uint32_t *__restrict__ rec_words,
                                                             const uint32_t *__restrict__ rec_esc,
                                                             uint8_t *out, uint64_t chunks_off,
                                                             const uint32_t *flags, int coder, uint32_t ce) {
    if (*flags) return;
    const uint32_t c = blockIdx.x;
    const uint32_t W = rec_words[c];
    const uint32_t start16 = reinterpret_cast<const uint32_t *>(out + kXcTabOff)[c];
    uint8_t *dst = out + chunks_off + 16ull * start16;
    const uint8_t *slot = slots + static_cast<uint64_t>(c) * slot_b;
    if (threadIdx.x < 32)
        reinterpret_cast<uint32_t *>(dst)[threadIdx.x] = reinterpret_cast<const uint32_t *>(slot)[threadIdx.x];
    // pair records: [states][n_words][n_esc][0][0][words][escapes]; rANS and
    // tANS records: [states][words]; zero-padded to 16 bytes.  rANS and pair
    // words sit at the end of the slot (written backwards), tANS words right
    // after the lane states; pair escapes end at hdr + ce (written backwards).
    const bool pair = coder == BS_CODER_RANS_PAIR;
    const uint32_t hdr = pair ? kXcPairRecHdr : 128u;
    const uint32_t E = pair ? rec_esc[c] : 0u;
    if (pair && threadIdx.x == 0) {
        uint32_t *d32 = reinterpret_cast<uint32_t *>(dst);
        d32[32] = W; d32[33] = E; d32[34] = 0; d32[35] = 0;
    }
    const uint8_t *ws = coder == BS_CODER_TANS ? slot + 128 : slot + slot_b - 2ull * W;
    const uint8_t *es = slot + hdr + ce - E;
    // body = words, escapes, zero pad: 16 bytes per thread and pass, shifted
    // from aligned 16-byte loads of the source region they lie in (words start
    // 2-byte aligned, escapes anywhere); the piece across the words/escapes
    // edge and the pad go 32 bits, then bytes, at a time
    const uint32_t wb = 2u * W, eb = wb + E;
    const uint32_t body = ((hdr + eb + 15u) & ~15u) - hdr;
    uint4 *bd = reinterpret_cast<uint4 *>(dst + hdr);
    for (uint32_t v = threadIdx.x; v < body / 16; v += blockDim.x) {
        const uint32_t j0 = 16 * v;
        if (j0 + 16 <= wb) {
            bd[v] = ld_u128_any(ws + j0);
            continue;
        }
        if (j0 >= wb && j0 + 16 <= eb) {
            bd[v] = ld_u128_any(es + (j0 - wb));
            continue;
        }
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t jb = 16 * v + 4 * k;
            if (jb + 4 <= wb) {
                o[k] = ld_u32_any(ws + jb);
            } else if (jb >= wb && jb + 4 <= eb) {
                o[k] = ld_u32_any(es + (jb - wb));
            } else {   // a piece across a region edge, or the pad
                uint32_t w = 0;
                for (uint32_t q = 0; q < 4; q++) {
                    const uint32_t b = jb + q;
                    const uint32_t byte = b < wb ? ws[b] : (b < eb ? es[b - wb] : 0u);
                    w |= byte << (8 * q);
                }
                o[k] = w;
            }
        }
        bd[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

cudaError_t launch_xc_encode(const uint16_t *d_in, uint64_t n, int coder, int prec, uint32_t ce, uint32_t groups,
                             uint8_t *d_out, uint64_t out_cap, uint64_t *d_out_len, uint8_t *d_ws,
                             uint64_t ws_bytes, cudaStream_t s) {
    const uint64_t nc = (n + ce - 1) / ce;
    auto *counts = reinterpret_cast<unsigned long long *>(d_ws + kWsCounts);
    auto *tab = reinterpret_cast<uint32_t *>(d_ws + kWsTab);
    auto *rcp = reinterpret_cast<const uint4 *>(d_ws + kWsRcp);
    auto *flags = reinterpret_cast<uint32_t *>(d_ws + kWsFlags);
    auto *aux = reinterpret_cast<uint32_t *>(d_ws + kWsAux);
    auto *recw = reinterpret_cast<uint32_t *>(d_ws + kWsRec);
    auto *rece = recw + nc;
    uint8_t *slots = d_ws + slots_off(nc);
    const uint64_t sb = slot_bytes(ce);
    const uint64_t plane_off = rup(kXcTabOff + 4 * (nc + 1), 16);
    const uint64_t chunks_off = plane_off + rup(n, 16);
    cudaError_t e = cudaMemsetAsync(counts, 0, 2048, s);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const bool pair = coder == BS_CODER_RANS_PAIR;
    const uint64_t vecs = pair && n >= kSampleMin ? sampled_vectors(n / 8) : n / 8;
    uint64_t want = (vecs + 255) / 256;
    int grid = static_cast<int>(want < static_cast<uint64_t>(sms) * 8 ? (want ? want : 1) : static_cast<uint64_t>(sms) * 8);
    uint16_t *slot_list = reinterpret_cast<uint16_t *>(d_ws + slotlist_off(nc));
    if (pair)
        xc_enc_expo_hist_kernel<<<grid, 256, 0, s>>>(d_in, n, counts);
    else
        xc_enc_hist_kernel<<<grid, 256, 0, s>>>(d_in, n, counts, d_out + plane_off);
    xc_enc_setup_kernel<<<1, 256, 0, s>>>(counts, d_in, n, coder, prec, ce, static_cast<uint32_t>(nc), groups, d_out,
                                          tab, slot_list, aux);
    const unsigned enc_blocks = static_cast<unsigned>((nc + kEncWarps - 1) / kEncWarps);
    if (coder == BS_CODER_RANS_PAIR) {
        xc_enc_chunks_pair_kernel<<<enc_blocks, kEncWarps * 32, 0, s>>>(d_in, n, ce, static_cast<uint32_t>(nc),
                                                                       rcp, aux, slots, sb, recw, rece,
                                                                       d_out + plane_off);
    } else if (coder == BS_CODER_TANS) {
        auto *scr = reinterpret_cast<uint32_t *>(d_ws + tans_scratch_off(nc, ce));
        xc_enc_chunks_tans_kernel<<<enc_blocks, kEncWarps * 32, 0, s>>>(d_in, n, ce, static_cast<uint32_t>(nc), prec,
                                                                       tab, slot_list, slots, sb, scr, recw);
    } else {
        xc_enc_chunks_kernel<<<enc_blocks, kEncWarps * 32, 0, s>>>(d_in, n, ce, static_cast<uint32_t>(nc),
                                                                  rcp, slots, sb, recw);
    }
    xc_enc_scan_kernel<<<1, 1024, 0, s>>>(recw, rece, coder, static_cast<uint32_t>(nc), d_out, chunks_off, out_cap,
                                          reinterpret_cast<unsigned long long *>(d_out_len), flags);
    xc_enc_compact_kernel<<<static_cast<unsigned>(nc), 256, 0, s>>>(slots, sb, recw, rece, d_out, chunks_off,
                                                                    flags, coder, ce);
    (void)ws_bytes;
    return cudaGetLastError();
}

}  // namespace bsg
