// xc_decode.cu -- sm_100a decoder of bf16_exp_chunked_v1 tensors.
//
// Format (this project's; the reference has no chunked codec -- its bf16
// codecs code the joint (sign,exponent) symbol serially, e.g.
// bigsmall/codecs/single_kernel.py:194-428):
//   * the 8-bit exponent of every bf16 value is entropy coded, rANS (32-bit
//     state, L = 2^16, 16-bit renorm, M = 2^P) or tANS (table of 2^P states);
//   * sign and mantissa are kept raw as one byte per value, (s << 7) | m, in a
//     byte plane that is merged back with 16-byte vector loads/stores;
//   * the tensor is cut into chunks of chunk_elems values; each chunk is one
//     "state group": 32 interleaved coder states (one per lane of a warp)
//     sharing one u16 word stream stored in consumption order.  Lane l owns
//     chunk elements g*256 + l*8 + j (group g, sub-step j < 8), so after 8
//     steps a lane holds 8 consecutive values and writes them as one 16-byte
//     store.  At each step the lanes needing a word take them in lane order:
//     word index = base + popc(ballot & lanemask_lt)  (Giesen's interleaved
//     rANS construction with a warp-shared stream).
//
// Kernels:
//   xc_prepare_kernel  one CTA per tensor: validates the blob header against the
//                      plan descriptor, builds the 2^P-entry decode table into
//                      the plan's workspace and checks the chunk offset table.
//   xc_decode_kernel   one CTA per work item (<= 16 chunks of one tensor): copies
//                      the table into shared memory, then each warp decodes one
//                      chunk.  Compressed words are staged per warp in a 2 KiB
//                      shared-memory ring (plus a 1 KiB mirror of its head)
//                      fed by 16-byte cp.async copies; the sign/mantissa plane
//                      is read with 8-byte loads two groups ahead; output
//                      leaves as 16-byte streaming stores.
#include <cstdint>
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace bsg {

// A work item is up to kWarps chunks of one tensor; the pair kernel runs one
// warp per chunk (16 warps share one staged 32 KiB table); the rANS/tANS
// kernel runs two CTAs of kRansWarps warps per item, one per half.
constexpr int kWarps = 16;                  // chunks per work item = warps per pair-kernel CTA
constexpr int kThreads = kWarps * 32;
constexpr int kRansWarps = 8;               // warps per rANS/tANS CTA
constexpr int kRansThreads = kRansWarps * 32;
constexpr int kRansMinBlocks = 5;           // 5 x 8 warps per SM: registers capped at 48
constexpr uint32_t kRingBytes = 2048;       // per-warp staging ring
constexpr uint32_t kFill = 512;             // bytes per refill: 32 lanes x 16 B

int xc_warps_per_cta() { return kWarps; }

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    // records are read front to back: ask L2 to fill 256 bytes per miss
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }
// wait until at most `pending` (0..3) of this thread's newest copy groups are in flight
__device__ __forceinline__ void cp_async_wait_pending(uint32_t pending) {
    switch (pending) {
        case 0: asm volatile("cp.async.wait_group 0;\n" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;\n" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;\n" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 3;\n" ::: "memory"); break;
    }
}

__device__ __forceinline__ uint2 ld_plane8(const uint8_t *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ void st_out16(uint16_t *p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// --------------------------------------------------------------------------
// table build
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) xc_prepare_kernel(XcTensorDev *tens, uint32_t *tables,
                                                         uint32_t *errs) {
    const int t = blockIdx.x;
    const int tid = threadIdx.x;
    XcTensorDev &T = tens[t];
    __shared__ uint32_t s_err, s_prec, s_coder, s_aux;
    __shared__ uint64_t s_chunks_off, s_plane_off, s_total;
    __shared__ uint32_t s_freq[256], s_cum[257];
    __shared__ uint32_t s_next[256];
    __shared__ uint8_t s_spread[kXcMaxTable];
    const uint8_t *b = T.blob;
    // the frequency table is loaded by every thread up front, its latency
    // overlapping the header checks (the check below guarantees it is in bounds)
    const bool hdr_in = T.blob_bytes >= kXcTabOff && !(reinterpret_cast<uintptr_t>(b) & 15);
    const uint32_t f = hdr_in ? reinterpret_cast<const uint16_t *>(b + kXcFreqOff)[tid] : 0u;
    if (tid == 0) {
        uint32_t err = 0;
        if (!hdr_in) {
            err = BS_DEV_HEADER;
        } else {
            const uint32_t *h32 = reinterpret_cast<const uint32_t *>(b);
            const uint64_t *h64 = reinterpret_cast<const uint64_t *>(b);
            uint32_t ver_coder_prec = h32[1];
            uint32_t ver = ver_coder_prec & 0xFFFF, coder = (ver_coder_prec >> 16) & 0xFF;
            uint32_t prec = ver_coder_prec >> 24;
            uint64_t n = h64[1];
            uint32_t ce = h32[4], nc = h32[5], lanes = h32[6], aux = h32[7];
            uint64_t co = h64[4], po = h64[5], total = h64[6];
            // the offset table has one entry per group (T.n_chunks) plus one
            const uint64_t po_want = (kXcTabOff + 4ull * (T.n_chunks + 1ull) + 15) & ~15ull;
            // version 1: one group per chunk; version 2: G groups per chunk
            const uint32_t G = ver == 2 ? h32[14] : 1u;
            const uint64_t ce_want = static_cast<uint64_t>(T.chunk_elems) * T.groups;
            const bool groups_ok = (ver == 1 && T.groups == 1) ||
                                   (ver == 2 && G == T.groups && h32[15] == 0);
            if (h32[0] != kXcMagic || !groups_ok || coder > 2 || prec < 8 || prec > 12 || n != T.n ||
                ce != ce_want || nc != (n + ce_want - 1) / ce_want || lanes != kXcLanes || po != po_want ||
                co != po + ((n + 15) & ~15ull) || total < co || (total & 15) || total > T.blob_bytes ||
                (coder == 2 ? aux > 241 : aux != 0) ||
                (T.coder_mask != 0 && coder <= 2 && !((T.coder_mask >> coder) & 1u)))
                err = BS_DEV_HEADER;
            s_total = total;
            s_prec = prec;
            s_coder = coder;
            s_aux = aux;
            s_chunks_off = co;
            s_plane_off = po;
        }
        s_err = err;
    }
    __syncthreads();
    if (s_err) {
        if (tid == 0) {
            errs[t] = s_err;
            T.coder = 0xFFFFFFFFu;
        }
        return;
    }
    const uint32_t P = s_prec, M = 1u << P, coder = s_coder;
    // frequencies and their exclusive prefix sum
    s_freq[tid] = f;
    __syncthreads();
    if (tid < 32) {
        // warp scan over 256 entries, 8 per lane
        uint32_t loc[8], sum = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            loc[k] = sum;
            sum += s_freq[tid * 8 + k];
        }
        uint32_t incl = sum;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            uint32_t v = __shfl_up_sync(kFull, incl, d);
            if (tid >= d) incl += v;
        }
        uint32_t excl = incl - sum;
#pragma unroll
        for (int k = 0; k < 8; k++) s_cum[tid * 8 + k] = excl + loc[k];
        if (tid == 31) s_cum[256] = incl;
    }
    __syncthreads();
    if (s_cum[256] != M || (coder != 1 && f >= M)) {
        if (tid == 0 || f >= M) atomicOr(&s_err, BS_DEV_FREQ);
    }
    __syncthreads();
    if (s_err) {
        if (tid == 0) {
            errs[t] = s_err;
            T.coder = 0xFFFFFFFFu;
        }
        return;
    }
    uint32_t *tab = tables + static_cast<uint64_t>(t) * kXcTableWords;
    if (coder == 2) {
        // pair entry (8 bytes): x = (slot - cum) | freq << 16; y = the two
        // exponents pre-shifted to their bf16 positions (e_a << 7 | e_b << 23),
        // with bit 15 / bit 31 flagging an escape (exponent in the record)
        const uint32_t per = (M + 255) / 256;
        const uint32_t s0 = tid * per, e_lo = s_aux;
        if (s0 < M) {
            int lo = 0, hi = 255;
            while (lo < hi) {
                int mid = (lo + hi + 1) >> 1;
                if (s_cum[mid] <= s0) lo = mid; else hi = mid - 1;
            }
            uint32_t s = lo;
            uint2 *tab2 = reinterpret_cast<uint2 *>(tab);
            for (uint32_t k = 0; k < per && s0 + k < M; k++) {
                const uint32_t slot = s0 + k;
                while (s_cum[s + 1] <= slot) s++;
                const uint32_t a = s >> 4, b = s & 15;
                const uint32_t y = (a == 15 ? 0x8000u : (e_lo + a) << 7) | (b == 15 ? 0x80000000u : (e_lo + b) << 23);
                tab2[slot] = make_uint2((slot - s_cum[s]) | (s_freq[s] << 16), y);
            }
        }
    } else if (coder == 0) {
        // rANS entry: (slot - cum) | sym << 12 | freq << 20; 16 slots per thread
        const uint32_t per = (M + 255) / 256;
        uint32_t s0 = tid * per;
        if (s0 < M) {
            int lo = 0, hi = 255;   // largest s with cum[s] <= s0
            while (lo < hi) {
                int mid = (lo + hi + 1) >> 1;
                if (s_cum[mid] <= s0) lo = mid; else hi = mid - 1;
            }
            uint32_t s = lo;
            for (uint32_t k = 0; k < per && s0 + k < M; k++) {
                uint32_t slot = s0 + k;
                while (s_cum[s + 1] <= slot) s++;
                tab[slot] = (slot - s_cum[s]) | (s << 12) | (s_freq[s] << 20);
            }
        }
    } else {
        // tANS: spread symbol occurrences with Collet's step, then give each
        // slot (in increasing order) its next state value x in [f, 2f)
        const uint32_t step = (M >> 1) + (M >> 3) + 3, mask = M - 1;
        for (uint32_t k = tid; k < M; k += blockDim.x) {
            int lo = 0, hi = 255;
            while (lo < hi) {
                int mid = (lo + hi + 1) >> 1;
                if (s_cum[mid] <= k) lo = mid; else hi = mid - 1;
            }
            s_spread[(k * step) & mask] = static_cast<uint8_t>(lo);
        }
        s_next[tid] = s_freq[tid];
        __syncthreads();
        if (tid < 32) {
            const uint32_t lt = lanemask_lt();
            for (uint32_t i0 = 0; i0 < M; i0 += 32) {
                uint32_t i = i0 + tid;
                uint32_t s = s_spread[i];
                uint32_t grp = __match_any_sync(kFull, s);
                uint32_t xs = s_next[s] + __popc(grp & lt);
                __syncwarp();
                if ((grp & lt) == 0) s_next[s] += __popc(grp);
                __syncwarp();
                uint32_t nb = P - (31 - __clz(xs));
                uint32_t base = (xs << nb) - M;
                tab[i] = base | (s << 12) | (nb << 20);
            }
        }
    }
    // The chunk offset table is checked where it is read: each decoding warp
    // checks its own chunk's two entries (checked_rec_bytes), so a plan that
    // decodes part of a tensor reads only its part of the table.
    if (tid == 0) {
        const uint64_t lim16 = (s_total - s_chunks_off) >> 4;
        errs[t] = 0;
        T.coder = coder;
        T.prec = P;
        T.chunks_off = s_chunks_off;
        T.plane_off = s_plane_off;
        T.aux = s_aux;
        T.rec_lim16 = lim16 > 0xFFFFFFFFull ? 0xFFFFFFFFu : static_cast<uint32_t>(lim16);
    }
}

// Record bytes of a chunk whose offset table entries are [a, z) (16-byte
// units from chunks_off), or 0 when the entries are not monotone with at least
// 128 bytes (the lane states) per record ending inside the record area.  The
// decode routines read nothing of a record whose size is 0.
__device__ __forceinline__ uint32_t checked_rec_bytes(uint32_t a, uint32_t z, uint32_t lim16) {
    return (z >= a && z - a >= 8 && z <= lim16) ? 16u * (z - a) : 0u;
}

// --------------------------------------------------------------------------
// chunk decode
// --------------------------------------------------------------------------
// Per-warp staging ring: kRingBytes of compressed words followed by a kMirror
// copy of the ring's first two kFill blocks.  One loop iteration (two groups of
// 8 steps) consumes at most 16 x 32 words = 1024 bytes, so reading from the
// iteration's start offset onwards never needs a wrap mask: offsets past
// kRingBytes land in the mirror.
constexpr uint32_t kMirror = 2 * kFill;
constexpr uint32_t kWarpRing = kRingBytes + kMirror;

struct Ring {
    uint8_t *buf;            // this warp's kWarpRing bytes of shared memory
    const uint8_t *src;      // first renorm word of the chunk record
    uint32_t bytes;          // renorm bytes in the record (multiple of 16)
    uint32_t fetched;        // bytes requested so far (multiple of kFill)
    uint32_t landed;         // bytes known to be in shared memory
};

__device__ __forceinline__ void ring_issue(Ring &r, uint32_t lane) {
    const uint32_t off = r.fetched + 16 * lane;
    if (off < r.bytes) {
        const uint32_t pos = off & (kRingBytes - 1);
        cp_async16(r.buf + pos, r.src + off);
        if (pos < kMirror) cp_async16(r.buf + kRingBytes + pos, r.src + off);
    }
    cp_async_commit();
    r.fetched += kFill;
}

// make bytes [0, min(bytes, consumed + kMirror)) visible to the whole warp
__device__ __forceinline__ void ring_ensure(Ring &r, uint32_t consumed_bytes) {
    uint32_t need = consumed_bytes + kMirror;
    if (need > r.bytes) need = r.bytes;
    if (need > r.landed) {
        cp_async_wait_all();
        __syncwarp();
        r.landed = r.fetched;
    }
}

// top up the ring after a group: one kFill refill if its slot is consumed
__device__ __forceinline__ void ring_refill(Ring &r, uint32_t consumed_bytes, uint32_t lane) {
    if (r.fetched < r.bytes && r.fetched + kFill - consumed_bytes <= kRingBytes) {
        __syncwarp();
        ring_issue(r, lane);
    }
}

// Decode-table entries keep the exponent symbol in bits 12..19:
//   rANS: (slot - cum) | sym << 12 | freq << 20
//   tANS: next-state base | sym << 12 | bits << 20
// Two bf16 words from two entries and the pair's sign|mantissa bytes given
// duplicated as [c0, c0, c1, c1]: bit 15/31 and bits 0-6/16-22 come from the
// plane bytes, bits 7-14/23-30 from the symbols.
__device__ __forceinline__ uint32_t merge_pair(uint32_t t0, uint32_t t1, uint32_t cc) {
    const uint32_t e7 = __byte_perm(t0, t1, 0x6521) << 3;
    return (cc & 0x807F807Fu) | (e7 & 0x7F807F80u);
}

__device__ __forceinline__ uint16_t merge_one(uint32_t t, uint32_t c) {
    return static_cast<uint16_t>(((c & 0x80u) << 8) | (((t >> 12) & 0xFFu) << 7) | (c & 0x7Fu));
}

template <int CODER>
__device__ __forceinline__ void decode_chunk(const uint32_t *__restrict__ s_tab, uint8_t *ring_buf,
                                             const uint8_t *__restrict__ rec, uint32_t rec_bytes,
                                             const uint8_t *__restrict__ plane,
                                             uint16_t *__restrict__ out, uint32_t cn, uint32_t P,
                                             uint32_t *err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t lt = lanemask_lt();
    const uint32_t smask = (1u << P) - 1;

    if (rec_bytes == 0) {   // bad chunk offset table entry
        if (lane == 0) atomicOr(err, BS_DEV_CHUNK_TABLE);
        return;
    }
    const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring_buf));
    const uint32_t tab_s = static_cast<uint32_t>(__cvta_generic_to_shared(s_tab));
    const uint32_t init = reinterpret_cast<const uint32_t *>(rec)[lane];
    // coder state: rANS x; tANS (st, bits, cnt)
    uint32_t x = init, st = init & 0xFFFF, bits = init >> 16, cnt = 16;
    (void)st; (void)bits; (void)cnt;

    Ring r{ring_buf, rec + 128, rec_bytes - 128, 0, 0};
#pragma unroll
    for (int k = 0; k < (int)(kRingBytes / kFill); k++) ring_issue(r, lane);

    uint32_t raddr = ring_s;  // shared address of the next unconsumed word (uniform)
    uint32_t consumed = 0;    // renorm bytes consumed so far (uniform)
    const uint32_t G = cn >> 8, rem = cn & 255;

    // One step for the whole warp; returns the lane's decode-table entry.  The
    // renorm word is read by every lane (inside the ring + mirror) and used
    // only where needed, so the step has no divergent branch.  Shared loads use
    // 32-bit shared-window addresses.
    auto step = [&](bool active) -> uint32_t {
        uint32_t t;
        if (CODER == 0) {
            t = lds_u32(tab_s + ((x & smask) << 2));
            const uint32_t nx = (t >> 20) * (x >> P) + (t & 0xFFFu);
            if (active) x = nx;
            const bool need = active && (x < kRansL);
            const uint32_t m = __ballot_sync(kFull, need);
            const uint32_t w = lds_u16(raddr + 2 * __popc(m & lt));
            if (need) x = x * 65536u + w;
            raddr += 2 * __popc(m);
        } else {
            const bool need = active && (cnt < P);
            const uint32_t m = __ballot_sync(kFull, need);
            const uint32_t w = lds_u16(raddr + 2 * __popc(m & lt));
            if (need) {
                bits |= w << cnt;
                cnt += 16;
            }
            raddr += 2 * __popc(m);
            t = lds_u32(tab_s + (st << 2));
            if (active) {
                const uint32_t nb = t >> 20;
                st = (t & 0xFFFu) + (bits & ((1u << nb) - 1));
                bits >>= nb;
                cnt -= nb;
            }
        }
        return t;
    };
    auto group = [&](uint32_t g, uint2 sm) {
        const uint32_t t0 = step(true), t1 = step(true), t2 = step(true), t3 = step(true);
        const uint32_t t4 = step(true), t5 = step(true), t6 = step(true), t7 = step(true);
        uint4 v;
        v.x = merge_pair(t0, t1, __byte_perm(sm.x, 0, 0x1100));
        v.y = merge_pair(t2, t3, __byte_perm(sm.x, 0, 0x3322));
        v.z = merge_pair(t4, t5, __byte_perm(sm.y, 0, 0x1100));
        v.w = merge_pair(t6, t7, __byte_perm(sm.y, 0, 0x3322));
        st_out16(out + g * 256 + lane * 8, v);
    };
    const uint32_t ring_end = ring_s + kRingBytes;
    const uint8_t *pl = plane + lane * 8;
    uint2 sm_a = make_uint2(0, 0), sm_b = make_uint2(0, 0);
    if (G > 0) sm_a = ld_plane8(pl);
    if (G > 1) sm_b = ld_plane8(pl + 256);
    uint32_t g = 0;
    for (; g + 1 < G; g += 2) {
        ring_ensure(r, consumed);
        if (raddr >= ring_end) raddr -= kRingBytes;
        const uint32_t rstart = raddr;
        const uint2 s0 = sm_a, s1 = sm_b;
        // next two groups' plane bytes (clamped to the last full group)
        sm_a = ld_plane8(pl + min(g + 2, G - 1) * 256);
        sm_b = ld_plane8(pl + min(g + 3, G - 1) * 256);
        group(g, s0);
        group(g + 1, s1);
        consumed += raddr - rstart;
        ring_refill(r, consumed, lane);
        ring_refill(r, consumed, lane);
    }
    if (g < G) {
        ring_ensure(r, consumed);
        if (raddr >= ring_end) raddr -= kRingBytes;
        const uint32_t rstart = raddr;
        group(g, sm_a);
        consumed += raddr - rstart;
    }
    if (rem) {
        ring_ensure(r, consumed);
        if (raddr >= ring_end) raddr -= kRingBytes;
        const uint32_t rstart = raddr;
        const uint32_t e_base = G * 256 + lane * 8;
#pragma unroll 1
        for (uint32_t j = 0; j < 8; j++) {
            const bool active = (lane * 8 + j) < rem;
            const uint32_t t = step(active);
            if (active) out[e_base + j] = merge_one(t, plane[e_base + j]);
        }
        consumed += raddr - rstart;
    }
    cp_async_wait_all();
    __syncwarp();
    const bool bad_state = CODER == 0 ? (x != kRansL) : (st != 0);
    const bool bad_stream = consumed > r.bytes || (r.bytes - consumed) >= 16;
    uint32_t code = (bad_state ? BS_DEV_FINAL_STATE : 0u) | (bad_stream ? BS_DEV_STREAM : 0u);
    code = __reduce_or_sync(kFull, code);
    if (code && lane == 0) atomicOr(err, code);
}

// --------------------------------------------------------------------------
// coder 2: rANS over exponent pairs.  One step decodes the two consecutive
// values a lane writes into one 32-bit output word, so a lane's 8 values take
// 4 steps.  The 8-byte table entry gives the state update (x) and both
// exponents already in their bf16 bit positions (y); a rare escape (bit 15 /
// bit 31 of y) takes its exponent from the record's escape list in a
// warp-uniform fix-up path.
// --------------------------------------------------------------------------
constexpr uint32_t kPairRingBytes = 2048;                // per-warp staging ring (power of 2)
constexpr uint32_t kPairMirror = kFill;                 // 8 pair-steps consume <= 512 B
constexpr uint32_t kPairWarpRing = kPairRingBytes + kPairMirror;
constexpr uint32_t kPairTableBytes = 8 * kXcMaxTable;
constexpr int kPairMinBlocks = 2;                        // CTAs (of kThreads) per SM the registers must allow

__device__ __forceinline__ uint2 lds_u64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

__device__ __forceinline__ void pair_ring_issue(Ring &r, uint32_t lane) {
    const uint32_t off = r.fetched + 16 * lane;
    if (off < r.bytes) {
        const uint32_t pos = off & (kPairRingBytes - 1);
        cp_async16(r.buf + pos, r.src + off);
        if (pos < kPairMirror) cp_async16(r.buf + kPairRingBytes + pos, r.src + off);
    }
    cp_async_commit();
    r.fetched += kFill;
}

__device__ __forceinline__ void pair_ring_ensure(Ring &r, uint32_t consumed_bytes) {
    uint32_t need = consumed_bytes + kPairMirror;
    if (need > r.bytes) need = r.bytes;
    if (need > r.landed) {
        // one copy group per kFill bytes, committed in order: the newest
        // (fetched - need) / kFill groups may stay in flight
        uint32_t pending = r.fetched > need ? (r.fetched - need) / kFill : 0u;
        if (pending > 3) pending = 3;
        cp_async_wait_pending(pending);
        __syncwarp();
        r.landed = r.fetched - pending * kFill;
    }
}

__device__ __forceinline__ void pair_ring_refill(Ring &r, uint32_t consumed_bytes, uint32_t lane) {
    if (r.fetched < r.bytes && r.fetched + kFill - consumed_bytes <= kPairRingBytes) {
        __syncwarp();
        pair_ring_issue(r, lane);
    }
}

// patch escaped exponents of one output word; `pos` is the warp's next escape
__device__ __forceinline__ uint32_t pair_patch(uint32_t word, uint32_t y, bool valid_b, const uint8_t *esc,
                                               uint32_t n_esc, uint32_t &pos, uint32_t lt, uint32_t &bad) {
    const bool ea = (y & 0x8000u) != 0;
    const bool eb = valid_b && (y & 0x80000000u) != 0;
    const uint32_t ba = __ballot_sync(kFull, ea), bb = __ballot_sync(kFull, eb);
    const uint32_t pa = pos + __popc(ba & lt) + __popc(bb & lt);
    const uint32_t pb = pa + (ea ? 1u : 0u);
    if (ea) {
        if (pa < n_esc) word = (word & ~0x7F80u) | (static_cast<uint32_t>(esc[pa]) << 7);
        else bad = 1;
    }
    if (eb) {
        if (pb < n_esc) word = (word & ~0x7F800000u) | (static_cast<uint32_t>(esc[pb]) << 23);
        else bad = 1;
    }
    pos += __popc(ba) + __popc(bb);
    return word;
}

__device__ __forceinline__ uint32_t merge_pair2(uint32_t y, uint32_t cc) {
    return (cc & 0x807F807Fu) | (y & 0x7F807F80u);
}

__device__ __forceinline__ void decode_chunk_pair(uint32_t tab_s, uint8_t *ring_buf,
                                                  const uint8_t *__restrict__ rec, uint32_t rec_bytes,
                                                  const uint8_t *__restrict__ plane,
                                                  uint16_t *__restrict__ out, uint32_t cn, uint32_t P,
                                                  uint32_t *err) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t lt = lanemask_lt();
    const uint32_t smask = (1u << P) - 1;
    const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring_buf));
    if (rec_bytes < kXcPairRecHdr) {   // bad chunk offset table entry, or a record too short for its header
        if (lane == 0) atomicOr(err, rec_bytes ? BS_DEV_STREAM : BS_DEV_CHUNK_TABLE);
        return;
    }
    const uint32_t *rec32 = reinterpret_cast<const uint32_t *>(rec);
    uint32_t x = rec32[lane];
    const uint32_t n_words = rec32[32], n_esc = rec32[33];
    uint32_t bad = (rec32[34] | rec32[35]) != 0 ? 1u : 0u;
    const uint64_t body = static_cast<uint64_t>(kXcPairRecHdr) + 2ull * n_words + n_esc;
    if (body > rec_bytes || rec_bytes - body >= 16) bad = 1;
    if (__any_sync(kFull, bad)) {
        if (lane == 0) atomicOr(err, BS_DEV_STREAM);
        return;
    }
    const uint8_t *esc = rec + kXcPairRecHdr + 2ull * n_words;
    // only the fix-up path reads the escape list, long after the chunk starts:
    // bring its first line into L1 now (lane 0, nothing waits on it)
    if (n_esc && lane == 0) asm volatile("prefetch.global.L1 [%0];" ::"l"(esc));
    uint32_t stage = (2 * n_words + 15) & ~15u;
    if (stage > rec_bytes - kXcPairRecHdr) stage = rec_bytes - kXcPairRecHdr;
    Ring r{ring_buf, rec + kXcPairRecHdr, stage, 0, 0};
#pragma unroll
    for (int k = 0; k < (int)(kPairRingBytes / kFill); k++) pair_ring_issue(r, lane);

    uint32_t raddr = ring_s, consumed = 0, epos = 0;
    const uint32_t G = cn >> 8, rem = cn & 255;

    auto step = [&](bool active) -> uint32_t {
        const uint2 t = lds_u64(tab_s + ((x & smask) << 3));
        const uint32_t nx = (t.x >> 16) * (x >> P) + (t.x & 0xFFFFu);
        if (active) x = nx;
        const bool need = active && (x < kRansL);
        const uint32_t m = __ballot_sync(kFull, need);
        const uint32_t w = lds_u16(raddr + 2 * __popc(m & lt));
        if (need) x = x * 65536u + w;
        raddr += 2 * __popc(m);
        return t.y;
    };
    auto group = [&](uint32_t g, uint2 sm) {
        const uint32_t y0 = step(true), y1 = step(true), y2 = step(true), y3 = step(true);
        uint4 v;
        v.x = merge_pair2(y0, __byte_perm(sm.x, 0, 0x1100));
        v.y = merge_pair2(y1, __byte_perm(sm.x, 0, 0x3322));
        v.z = merge_pair2(y2, __byte_perm(sm.y, 0, 0x1100));
        v.w = merge_pair2(y3, __byte_perm(sm.y, 0, 0x3322));
        if (__any_sync(kFull, ((y0 | y1 | y2 | y3) & 0x80008000u) != 0)) {
            // patch only the pair-steps that hold an escape (a step without
            // one would add nothing to the escape position)
            if (__any_sync(kFull, (y0 & 0x80008000u) != 0)) v.x = pair_patch(v.x, y0, true, esc, n_esc, epos, lt, bad);
            if (__any_sync(kFull, (y1 & 0x80008000u) != 0)) v.y = pair_patch(v.y, y1, true, esc, n_esc, epos, lt, bad);
            if (__any_sync(kFull, (y2 & 0x80008000u) != 0)) v.z = pair_patch(v.z, y2, true, esc, n_esc, epos, lt, bad);
            if (__any_sync(kFull, (y3 & 0x80008000u) != 0)) v.w = pair_patch(v.w, y3, true, esc, n_esc, epos, lt, bad);
        }
        st_out16(out + g * 256 + lane * 8, v);
    };
    const uint32_t ring_end = ring_s + kPairRingBytes;
    const uint8_t *pl = plane + lane * 8;
    uint2 sm_a = make_uint2(0, 0), sm_b = make_uint2(0, 0);
    if (G > 0) sm_a = ld_plane8(pl);
    if (G > 1) sm_b = ld_plane8(pl + 256);
    uint32_t g = 0;
    for (; g + 1 < G; g += 2) {
        pair_ring_ensure(r, consumed);
        if (raddr >= ring_end) raddr -= kPairRingBytes;
        const uint32_t rstart = raddr;
        const uint2 s0 = sm_a, s1 = sm_b;
        sm_a = ld_plane8(pl + min(g + 2, G - 1) * 256);
        sm_b = ld_plane8(pl + min(g + 3, G - 1) * 256);
        group(g, s0);
        group(g + 1, s1);
        consumed += raddr - rstart;
        pair_ring_refill(r, consumed, lane);
    }
    if (g < G) {
        pair_ring_ensure(r, consumed);
        if (raddr >= ring_end) raddr -= kPairRingBytes;
        const uint32_t rstart = raddr;
        group(g, sm_a);
        consumed += raddr - rstart;
    }
    if (rem) {
        pair_ring_ensure(r, consumed);
        if (raddr >= ring_end) raddr -= kPairRingBytes;
        const uint32_t rstart = raddr;
        const uint32_t e_base = G * 256 + lane * 8;
#pragma unroll 1
        for (uint32_t jj = 0; jj < 4; jj++) {
            const uint32_t e = lane * 8 + 2 * jj;
            const bool active = e < rem;
            const bool second = e + 1 < rem;
            const uint32_t y = step(active);
            uint32_t c0 = active ? plane[e_base + 2 * jj] : 0u, c1 = second ? plane[e_base + 2 * jj + 1] : 0u;
            uint32_t word = merge_pair2(y, c0 | (c0 << 8) | (c1 << 16) | (c1 << 24));
            if (__any_sync(kFull, active && (y & (second ? 0x80008000u : 0x8000u)) != 0))
                word = pair_patch(word, active ? y : 0u, second, esc, n_esc, epos, lt, bad);
            if (active) out[e_base + 2 * jj] = static_cast<uint16_t>(word);
            if (second) out[e_base + 2 * jj + 1] = static_cast<uint16_t>(word >> 16);
        }
        consumed += raddr - rstart;
    }
    cp_async_wait_all();
    __syncwarp();
    const bool bad_state = x != kRansL;
    const bool bad_stream = consumed != 2 * n_words || epos != n_esc || bad;
    uint32_t code = (bad_state ? BS_DEV_FINAL_STATE : 0u) | (bad_stream ? BS_DEV_STREAM : 0u);
    code = __reduce_or_sync(kFull, code);
    if (code && lane == 0) atomicOr(err, code);
}

// Both decode kernels walk the work list with a grid stride, so a plan can
// cap its CTAs (bs_plan_set_max_ctas) and leave SM room to kernels on other
// streams; uncapped, the grid is one CTA per item and the loop runs once.
__global__ void __launch_bounds__(kThreads, kPairMinBlocks) xc_decode_pair_kernel(const XcTensorDev *__restrict__ tens,
                                                                  const XcItem *__restrict__ items, int n_items,
                                                                  const uint32_t *__restrict__ tables,
                                                                  uint32_t *errs) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *s_ring = smem + kPairTableBytes;
    const uint32_t warp = threadIdx.x >> 5;
    uint32_t staged = 0xFFFFFFFFu;   // tensor whose table is in shared memory
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const XcItem it = items[item];
        const XcTensorDev &T = tens[it.tensor];
        if (T.coder != 2) continue;   // other coders: xc_decode_kernel; flagged tensors: skipped
        const uint32_t P = T.prec;
        const uint32_t M = 1u << P;
        // this warp's chunk offsets, loaded before the table staging so the
        // two loads' latency hides behind it
        const bool mine = warp < it.n_chunks;
        const uint32_t c = it.first_chunk + warp;
        const uint8_t *blob = T.blob;
        const uint32_t *cs = reinterpret_cast<const uint32_t *>(blob + kXcTabOff);
        uint32_t a = 0, z = 0;
        if (mine) {
            a = cs[c];
            z = cs[c + 1];
        }
        if (it.tensor != staged) {    // a capped grid often walks several items of one tensor
            const uint4 *src =
                reinterpret_cast<const uint4 *>(tables + static_cast<uint64_t>(it.tensor) * kXcTableWords);
            __syncthreads();   // the previous item's warps are done with the table
            for (uint32_t i = threadIdx.x; i < M / 2; i += kThreads) reinterpret_cast<uint4 *>(smem)[i] = src[i];
            __syncthreads();
            staged = it.tensor;
        }
        if (!mine) continue;
        const uint64_t e0 = static_cast<uint64_t>(c) * T.chunk_elems;
        const uint64_t left = T.n - e0;
        const uint32_t cn = left < T.chunk_elems ? static_cast<uint32_t>(left) : T.chunk_elems;
        decode_chunk_pair(static_cast<uint32_t>(__cvta_generic_to_shared(smem)), s_ring + warp * kPairWarpRing,
                          blob + T.chunks_off + 16ull * a, checked_rec_bytes(a, z, T.rec_lim16), blob + T.plane_off + e0,
                          T.out + (e0 - static_cast<uint64_t>(T.chunk_begin) * T.chunk_elems), cn, P,
                          &errs[it.tensor]);
    }
}

__global__ void __launch_bounds__(kRansThreads, kRansMinBlocks) xc_decode_kernel(const XcTensorDev *__restrict__ tens,
                                                             const XcItem *__restrict__ items, int n_items,
                                                             const uint32_t *__restrict__ tables,
                                                             uint32_t *errs) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t *s_tab = reinterpret_cast<uint32_t *>(smem);
    uint8_t *s_ring = smem + kXcMaxTable * 4;
    const uint32_t warp = threadIdx.x >> 5;
    uint32_t staged = 0xFFFFFFFFu;   // tensor whose table is in shared memory
    for (int half = blockIdx.x; half < 2 * n_items; half += gridDim.x) {
        const XcItem it = items[half >> 1];
        const uint32_t k = (half & 1) * kRansWarps + warp;   // this warp's chunk within the item
        const XcTensorDev &T = tens[it.tensor];
        const uint32_t coder = T.coder;
        if (coder > 1) continue;   // the table build flagged this tensor, or the pair kernel's
        const uint32_t P = T.prec;
        const uint32_t M = 1u << P;
        const bool mine = k < it.n_chunks;   // chunk offsets loaded before the table staging
        const uint32_t c = it.first_chunk + k;
        const uint8_t *blob = T.blob;
        const uint32_t *cs = reinterpret_cast<const uint32_t *>(blob + kXcTabOff);
        uint32_t a = 0, z = 0;
        if (mine) {
            a = cs[c];
            z = cs[c + 1];
        }
        if (it.tensor != staged) {    // a capped grid often walks several items of one tensor
            const uint4 *src =
                reinterpret_cast<const uint4 *>(tables + static_cast<uint64_t>(it.tensor) * kXcTableWords);
            __syncthreads();   // the previous item's warps are done with the table
            for (uint32_t i = threadIdx.x; i < M / 4; i += kRansThreads) reinterpret_cast<uint4 *>(s_tab)[i] = src[i];
            __syncthreads();
            staged = it.tensor;
        }
        if (!mine) continue;
        const uint8_t *rec = blob + T.chunks_off + 16ull * a;
        const uint32_t rec_bytes = checked_rec_bytes(a, z, T.rec_lim16);
        const uint64_t e0 = static_cast<uint64_t>(c) * T.chunk_elems;
        const uint64_t left = T.n - e0;
        const uint32_t cn = left < T.chunk_elems ? static_cast<uint32_t>(left) : T.chunk_elems;
        uint8_t *ring = s_ring + warp * kWarpRing;
        const uint8_t *plane = blob + T.plane_off + e0;
        uint16_t *out = T.out + (e0 - static_cast<uint64_t>(T.chunk_begin) * T.chunk_elems);
        if (coder == 0)
            decode_chunk<0>(s_tab, ring, rec, rec_bytes, plane, out, cn, P, &errs[it.tensor]);
        else
            decode_chunk<1>(s_tab, ring, rec, rec_bytes, plane, out, cn, P, &errs[it.tensor]);
    }
}

cudaError_t launch_xc_prepare(XcTensorDev *d_tens, int n_tensors, uint32_t *d_tables, uint32_t *d_errs,
                              cudaStream_t s) {
    if (n_tensors <= 0) return cudaSuccess;
    xc_prepare_kernel<<<n_tensors, 256, 0, s>>>(d_tens, d_tables, d_errs);
    return cudaGetLastError();
}

// Dynamic shared-memory opt-in, once per (kernel, device): the attribute
// belongs to the module loaded in each device's context.
template <typename K>
static cudaError_t smem_opt_in(K kernel, size_t bytes, std::atomic<uint8_t> *done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) done[dev].store(1, std::memory_order_release);
    return e;
}
static std::atomic<uint8_t> g_attr_rans[128], g_attr_pair[128], g_attr_na_pair[128];

// The decode kernels' shared-memory opt-in for the coder families in
// `coders` (what launch_xc_decode does first), so a stream capture of
// launch_xc_decode records kernel launches only.
cudaError_t xc_decode_attrs(uint32_t coders) {
    cudaError_t e = cudaSuccess;
    if (coders & ((1u << BS_CODER_RANS) | (1u << BS_CODER_TANS)))
        e = smem_opt_in(xc_decode_kernel, kXcMaxTable * 4 + kRansWarps * kWarpRing, g_attr_rans);
    if (e == cudaSuccess && (coders & (1u << BS_CODER_RANS_PAIR)))
        e = smem_opt_in(xc_decode_pair_kernel, kPairTableBytes + kWarps * kPairWarpRing, g_attr_pair);
    return e;
}

uint32_t xc_launch_mask(const XcTensorDev *h_tens, int n) {
    uint32_t m = 0;
    for (int i = 0; i < n; i++) m |= h_tens[i].coder_mask ? h_tens[i].coder_mask : kXcAllCoders;
    return m;
}

// One launch per coder family present: coders 0/1 share xc_decode_kernel,
// coder 2 has its own.  A CTA whose tensor uses the other family (possible
// only with coder_mask 0) or was flagged by the prepare kernel returns at once.
cudaError_t launch_xc_decode(const XcTensorDev *d_tens, const XcItem *d_items, int n_items,
                             const uint32_t *d_tables, uint32_t *d_errs, uint32_t coders, int max_ctas,
                             cudaStream_t s) {
    if (n_items <= 0) return cudaSuccess;
    const int grid = max_ctas > 0 && max_ctas < n_items ? max_ctas : n_items;
    cudaError_t e = cudaSuccess;
    if (coders & ((1u << BS_CODER_RANS) | (1u << BS_CODER_TANS))) {
        const size_t smem = kXcMaxTable * 4 + kRansWarps * kWarpRing;
        e = smem_opt_in(xc_decode_kernel, smem, g_attr_rans);
        if (e != cudaSuccess) return e;
        // two CTAs per item (one per half of its chunks); a cap counts pair-kernel-sized CTAs
        const int rgrid = 2 * grid;
        xc_decode_kernel<<<rgrid, kRansThreads, smem, s>>>(d_tens, d_items, n_items, d_tables, d_errs);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (coders & (1u << BS_CODER_RANS_PAIR)) {
        const size_t psmem = kPairTableBytes + kWarps * kPairWarpRing;
        e = smem_opt_in(xc_decode_pair_kernel, psmem, g_attr_pair);
        if (e != cudaSuccess) return e;
        xc_decode_pair_kernel<<<grid, kThreads, psmem, s>>>(d_tens, d_items, n_items, d_tables, d_errs);
        e = cudaGetLastError();
    }
    return e;
}

// --------------------------------------------------------------------------
// Allocation-free decode (bs_xc_decode_noalloc).
//
// For callers that must not allocate device memory: the per-call scratch (the
// tensors' descriptors, their decode tables and status words) lives in this
// file-scope array instead of plan memory.  Every GPU that loads the library
// holds it (kNoallocScratchBytes) until the process exits.  All calls share
// it, so calls whose GPU work overlaps race; each call rewrites every field it
// reads (descriptors by the stage kernel, tables and status words by
// xc_prepare_kernel), so a call never depends on what the previous one left.
// --------------------------------------------------------------------------
constexpr int kNoallocMaxTensors = BS_NOALLOC_MAX_TENSORS;
constexpr uint64_t kNoallocTablesOff = 0;
constexpr uint64_t kNoallocTensOff = kNoallocTablesOff + 4ull * kXcTableWords * kNoallocMaxTensors;
constexpr uint64_t kNoallocErrsOff = kNoallocTensOff + 256ull * ((sizeof(XcTensorDev) * kNoallocMaxTensors + 255) / 256);
constexpr uint64_t kNoallocScratchBytes = kNoallocErrsOff + 256;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

// by-value kernel arguments: descriptors and the per-tensor CTA prefix
struct NoallocArgs {
    XcTensorDev tens[kNoallocMaxTensors];
    uint32_t range_count[kNoallocMaxTensors];        // chunks decoded per tensor
    uint32_t cta_prefix[kNoallocMaxTensors + 1];     // first CTA of each tensor
    int n;
};

__global__ void xc_noalloc_stage_kernel(const NoallocArgs a, XcTensorDev *tens) {
    const int t = threadIdx.x;
    if (t < a.n) tens[t] = a.tens[t];
}

__global__ void __launch_bounds__(kRansThreads, kRansMinBlocks) xc_decode_noalloc_kernel(const NoallocArgs a,
                                                                     const XcTensorDev *__restrict__ tens,
                                                                     const uint32_t *__restrict__ tables,
                                                                     uint32_t *errs) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t *s_tab = reinterpret_cast<uint32_t *>(smem);
    uint8_t *s_ring = smem + kXcMaxTable * 4;
    const uint32_t unit = blockIdx.x >> 1;   // two CTAs (halves) per kWarps-chunk unit
    int ti = 0;
    while (ti + 1 < a.n && unit >= a.cta_prefix[ti + 1]) ti++;
    const XcTensorDev &T = tens[ti];
    const uint32_t coder = T.coder;
    if (coder > 1) return;   // xc_prepare_kernel flagged this tensor
    const uint32_t P = T.prec;
    const uint32_t M = 1u << P;
    const uint4 *src = reinterpret_cast<const uint4 *>(tables + static_cast<uint64_t>(ti) * kXcTableWords);
    for (uint32_t i = threadIdx.x; i < M / 4; i += kRansThreads) reinterpret_cast<uint4 *>(s_tab)[i] = src[i];
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t c0 = a.tens[ti].chunk_begin;
    const uint32_t c = c0 + (unit - a.cta_prefix[ti]) * kWarps + (blockIdx.x & 1) * kRansWarps + warp;
    if (c >= c0 + a.range_count[ti]) return;
    const uint8_t *blob = T.blob;
    const uint32_t *cs = reinterpret_cast<const uint32_t *>(blob + kXcTabOff);
    const uint32_t ca = cs[c], cz = cs[c + 1];
    const uint8_t *rec = blob + T.chunks_off + 16ull * ca;
    const uint32_t rec_bytes = checked_rec_bytes(ca, cz, T.rec_lim16);
    const uint64_t e0 = static_cast<uint64_t>(c) * T.chunk_elems;
    const uint64_t left = T.n - e0;
    const uint32_t cn = left < T.chunk_elems ? static_cast<uint32_t>(left) : T.chunk_elems;
    uint8_t *ring = s_ring + warp * kWarpRing;
    const uint8_t *plane = blob + T.plane_off + e0;
    uint16_t *out = T.out + (e0 - static_cast<uint64_t>(T.chunk_begin) * T.chunk_elems);
    if (coder == 0)
        decode_chunk<0>(s_tab, ring, rec, rec_bytes, plane, out, cn, P, &errs[ti]);
    else
        decode_chunk<1>(s_tab, ring, rec, rec_bytes, plane, out, cn, P, &errs[ti]);
}

__global__ void __launch_bounds__(kThreads, kPairMinBlocks) xc_decode_noalloc_pair_kernel(const NoallocArgs a,
                                                                          const XcTensorDev *__restrict__ tens,
                                                                          const uint32_t *__restrict__ tables,
                                                                          uint32_t *errs) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *s_ring = smem + kPairTableBytes;
    int ti = 0;
    while (ti + 1 < a.n && blockIdx.x >= a.cta_prefix[ti + 1]) ti++;
    const XcTensorDev &T = tens[ti];
    if (T.coder != 2) return;
    const uint32_t P = T.prec;
    const uint32_t M = 1u << P;
    const uint4 *src = reinterpret_cast<const uint4 *>(tables + static_cast<uint64_t>(ti) * kXcTableWords);
    for (uint32_t i = threadIdx.x; i < M / 2; i += kThreads) reinterpret_cast<uint4 *>(smem)[i] = src[i];
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t c0 = a.tens[ti].chunk_begin;
    const uint32_t c = c0 + (blockIdx.x - a.cta_prefix[ti]) * kWarps + warp;
    if (c >= c0 + a.range_count[ti]) return;
    const uint8_t *blob = T.blob;
    const uint32_t *cs = reinterpret_cast<const uint32_t *>(blob + kXcTabOff);
    const uint32_t ca = cs[c], cz = cs[c + 1];
    const uint64_t e0 = static_cast<uint64_t>(c) * T.chunk_elems;
    const uint64_t left = T.n - e0;
    const uint32_t cn = left < T.chunk_elems ? static_cast<uint32_t>(left) : T.chunk_elems;
    decode_chunk_pair(static_cast<uint32_t>(__cvta_generic_to_shared(smem)), s_ring + warp * kPairWarpRing,
                      blob + T.chunks_off + 16ull * ca, checked_rec_bytes(ca, cz, T.rec_lim16), blob + T.plane_off + e0,
                      T.out + (e0 - static_cast<uint64_t>(T.chunk_begin) * T.chunk_elems), cn, P, &errs[ti]);
}

namespace {
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[128] = {};   // device address of g_noalloc_scratch, per device
}  // namespace

// Set-up (first call on a device, with that device current): resolve the
// scratch array's device address.  In host code the symbol is only a host-side
// stand-in, so kernels receive this address instead.
static cudaError_t noalloc_scratch(int dev, uint8_t **out) {
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = static_cast<uint8_t *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

cudaError_t launch_xc_noalloc(const XcTensorDev *h_tens, const uint32_t *range_count, int n, cudaStream_t s,
                              uint32_t *h_status) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    uint8_t *scr = nullptr;
    e = noalloc_scratch(dev, &scr);
    if (e != cudaSuccess) return e;
    XcTensorDev *d_tens = reinterpret_cast<XcTensorDev *>(scr + kNoallocTensOff);
    uint32_t *d_tables = reinterpret_cast<uint32_t *>(scr + kNoallocTablesOff);
    uint32_t *d_errs = reinterpret_cast<uint32_t *>(scr + kNoallocErrsOff);
    NoallocArgs a{};
    a.n = n;
    a.cta_prefix[0] = 0;
    for (int i = 0; i < n; i++) {
        a.tens[i] = h_tens[i];
        a.range_count[i] = range_count[i];
        a.cta_prefix[i + 1] = a.cta_prefix[i] + (range_count[i] + kWarps - 1) / kWarps;
    }
    for (int i = n; i < kNoallocMaxTensors; i++) a.cta_prefix[i + 1] = a.cta_prefix[n];
    xc_noalloc_stage_kernel<<<1, kNoallocMaxTensors, 0, s>>>(a, d_tens);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = launch_xc_prepare(d_tens, n, d_tables, d_errs, s);
    const uint32_t coders = xc_launch_mask(h_tens, n);
    if (e == cudaSuccess && a.cta_prefix[n] > 0 && (coders & ((1u << BS_CODER_RANS) | (1u << BS_CODER_TANS)))) {
        const size_t smem = kXcMaxTable * 4 + kRansWarps * kWarpRing;   // below the 48 KiB default
        xc_decode_noalloc_kernel<<<2 * a.cta_prefix[n], kRansThreads, smem, s>>>(a, d_tens, d_tables, d_errs);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && a.cta_prefix[n] > 0 && (coders & (1u << BS_CODER_RANS_PAIR))) {
        const size_t psmem = kPairTableBytes + kWarps * kPairWarpRing;
        e = smem_opt_in(xc_decode_noalloc_pair_kernel, psmem, g_attr_na_pair);
        if (e == cudaSuccess) {
            xc_decode_noalloc_pair_kernel<<<a.cta_prefix[n], kThreads, psmem, s>>>(a, d_tens, d_tables, d_errs);
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_status, d_errs, 4ull * n, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

uint64_t xc_noalloc_scratch_bytes() { return kNoallocScratchBytes; }

}  // namespace bsg
