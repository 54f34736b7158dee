// par_decode.cu -- sm_100a decoder of the reference's bf16_parallel_v1 format.
//
// The reference decodes this format with one Triton program per stream for the
// (sign,exp) substream only, then decodes every mantissa bucket, un-sorts and
// merges on the CPU (bigsmall/kernels/ac_triton.py:172-262).  Here everything
// stays on the device:
//   par_jobs_kernel   one CTA per serial rANS stream: every stream's SE
//                     substream and every (stream, exponent) mantissa bucket is
//                     an independent job, all decoded concurrently with the
//                     exact bigsmall/codecs/rans.py:165-207 state machine
//                     (including its end-of-data zero fill).  The same kernel
//                     runs the legacy serial formats' streams
//                     (bf16_se_single_kernel, bf16_se_tans: one SE stream per
//                     tensor plus one stream per exponent bucket).
//   par_merge_kernel  one warp per PAR1 stream (one per tensor for the legacy
//                     formats): rebuilds the stream's bucket starts
//                     from the decoded exponents (rans bincount/cumsum,
//                     bf16_parallel.py:318-321), checks them against the bucket
//                     counts recorded in the blob, and inverts the stable argsort
//                     (:328-344) 32 elements at a time with __match_any_sync
//                     ranks, writing bf16 (:349-352) at element k + i*n_streams.
#include <cstdint>

#include "common.cuh"

namespace bsg {

__device__ __forceinline__ uint32_t lanemask_lt_p() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

constexpr int kJobThreads = 32 * static_cast<int>(kJobGroup);

__device__ __forceinline__ uint2 lds_entry(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

__device__ __forceinline__ uint32_t lds_sym(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}

// The serial loop of one stream.  A single thread has no other work to hide
// latency behind, so the state's dependency chain per symbol is kept to: mask
// + shift for the slot address, one shared-memory load of {freq, slot - cum},
// one IMAD, and a compare-select renorm.  The symbol comes from a separate
// table load off that chain; the next renorm word is loaded as soon as the
// previous one is consumed; stores are off the chain.  SLOW adds the second
// renorm read the reference's while-loop performs when a step leaves the
// state below 2^16 twice (only possible from an initial state below L or a
// slot whose frequency is 0).
template <int PREC, bool SLOW, typename OutT>
__device__ __forceinline__ void serial_stream(uint32_t tab_s, uint32_t sym_s, const uint8_t *__restrict__ d,
                                              uint32_t avail, uint32_t n_words, uint32_t w, uint32_t state,
                                              uint32_t n_syms, OutT *__restrict__ out) {
    constexpr uint32_t kMask = (1u << PREC) - 1;
    const uint32_t n_full = min(n_words, avail >> 1);   // words with both bytes present
    auto word = [&](uint32_t k) -> uint32_t {
        const uint32_t i = 2 * k;
        if (k < n_full) return static_cast<uint32_t>(d[i]) | (static_cast<uint32_t>(d[i + 1]) << 8);
        return (i < avail ? static_cast<uint32_t>(d[i]) : 0u);   // odd tail byte, or a zero word
    };
    uint32_t next = w < n_words ? word(w) : 0u;
    auto step = [&]() -> uint32_t {
        const uint32_t slot = state & kMask;
        const uint2 e = lds_entry(tab_s + (slot << 3));
        const uint32_t sym = lds_sym(sym_s + (slot << 1));
        state = e.x * (state >> PREC) + e.y;
        const bool r = state < kRansL && w < n_words;
        state = r ? ((state << 16) | next) : state;
        if (r) {
            w++;
            next = w < n_words ? word(w) : 0u;
        }
        if (SLOW) {
            while (state < kRansL && w < n_words) {
                state = (state << 16) | next;
                w++;
                next = w < n_words ? word(w) : 0u;
            }
        }
        return sym;
    };
    uint32_t i = 0;
    for (; i + 4 <= n_syms; i += 4) {
        const uint32_t s0 = step(), s1 = step(), s2 = step(), s3 = step();
        out[i] = static_cast<OutT>(s0);
        out[i + 1] = static_cast<OutT>(s1);
        out[i + 2] = static_cast<OutT>(s2);
        out[i + 3] = static_cast<OutT>(s3);
    }
    for (; i < n_syms; i++) out[i] = static_cast<OutT>(step());
}

// One CTA per serial stream: the CTA stages the stream's decode tables
// (slot -> {freq, slot - cum} and slot -> symbol) in shared memory, then one
// thread runs the stream.  The state stays below 2^32 because the host rejects
// tables with a frequency above M, so 32-bit arithmetic is exact.
__global__ void __launch_bounds__(kJobThreads) par_jobs_kernel(const ParJob *__restrict__ jobs,
                                                               const uint2 *__restrict__ tabs,
                                                               const uint16_t *__restrict__ syms,
                                                               uint16_t *__restrict__ se_sym,
                                                               uint8_t *__restrict__ mant, uint32_t *errs) {
    extern __shared__ __align__(16) uint8_t s_mem[];
    uint2 *s_tab = reinterpret_cast<uint2 *>(s_mem);
    uint16_t *s_sym = reinterpret_cast<uint16_t *>(s_mem + 4096 * sizeof(uint2));
    const ParJob J = jobs[blockIdx.x];
    if (J.n_syms == 0) return;
    const bool is_se = (J.flags & kJobSe) != 0;
    const uint32_t M = is_se ? 4096u : 1024u;
    for (uint32_t i = threadIdx.x; i < M; i += kJobThreads) {
        s_tab[i] = tabs[J.tab_off + i];
        s_sym[i] = syms[J.tab_off + i];
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    const uint8_t *d = reinterpret_cast<const uint8_t *>(J.data);
    const uint32_t avail = J.avail, n_words = J.n_words;
    uint32_t state, w = 0;
    if (J.flags & kJobStateInStream) {
        if (n_words < 2) {   // rans.py:176-177 / numba_rans: a stream shorter than its state
            atomicOr(&errs[J.tensor], BS_DEV_STREAM);
            return;
        }
        auto word = [&](uint32_t k) -> uint32_t {
            const uint32_t i = 2 * k;
            return (i < avail ? static_cast<uint32_t>(d[i]) : 0u) |
                   (i + 1 < avail ? static_cast<uint32_t>(d[i + 1]) << 8 : 0u);
        };
        state = word(0) | (word(1) << 16);
        w = 2;
    } else {
        state = J.state0;
    }
    const uint32_t tab_s = static_cast<uint32_t>(__cvta_generic_to_shared(s_tab));
    const uint32_t sym_s = static_cast<uint32_t>(__cvta_generic_to_shared(s_sym));
    const bool slow = (J.flags & kJobSlowRenorm) != 0;
    if (is_se) {
        if (slow) serial_stream<12, true>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, se_sym + J.out_off);
        else serial_stream<12, false>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, se_sym + J.out_off);
    } else {
        if (slow) serial_stream<10, true>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, mant + J.out_off);
        else serial_stream<10, false>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, mant + J.out_off);
    }
}

// One CTA per group of up to kJobGroup serial streams that share a decode
// table (all slices of a bf16_parallel_v1 tensor share its (sign,exp) table
// and, per exponent, its mantissa table; a legacy stream has its own): the
// CTA stages the table (slot -> {freq, slot - cum} and slot -> symbol) in
// shared memory once, then one lane of each warp runs one stream (a stream
// per lane would diverge on every renorm).  The state stays below 2^32
// because the host rejects tables with a frequency above M, so 32-bit
// arithmetic is exact.
__global__ void __launch_bounds__(kJobThreads) par_groups_kernel(const ParJob *__restrict__ jobs,
                                                                 const uint2 *__restrict__ groups,
                                                               const uint2 *__restrict__ tabs,
                                                               const uint16_t *__restrict__ syms,
                                                               uint16_t *__restrict__ se_sym,
                                                               uint8_t *__restrict__ mant, uint32_t *errs) {
    extern __shared__ __align__(16) uint8_t s_mem[];
    uint2 *s_tab = reinterpret_cast<uint2 *>(s_mem);
    uint16_t *s_sym = reinterpret_cast<uint16_t *>(s_mem + 4096 * sizeof(uint2));
    const uint2 G = groups[blockIdx.x];   // {first job, jobs (<= kJobGroup)}
    const uint32_t warp = threadIdx.x >> 5;
    const bool runs = warp < G.y && (threadIdx.x & 31) == 0;
    const ParJob J = jobs[G.x + (warp < G.y ? warp : 0u)];   // every job of the group has the same table
    const bool is_se = (J.flags & kJobSe) != 0;
    const uint32_t M = is_se ? 4096u : 1024u;
    for (uint32_t i = threadIdx.x; i < M; i += kJobThreads) {
        s_tab[i] = tabs[J.tab_off + i];
        s_sym[i] = syms[J.tab_off + i];
    }
    __syncthreads();
    if (!runs || J.n_syms == 0) return;
    const uint8_t *d = reinterpret_cast<const uint8_t *>(J.data);
    const uint32_t avail = J.avail, n_words = J.n_words;
    uint32_t state, w = 0;
    if (J.flags & kJobStateInStream) {
        if (n_words < 2) {   // rans.py:176-177 / numba_rans: a stream shorter than its state
            atomicOr(&errs[J.tensor], BS_DEV_STREAM);
            return;
        }
        auto word = [&](uint32_t k) -> uint32_t {
            const uint32_t i = 2 * k;
            return (i < avail ? static_cast<uint32_t>(d[i]) : 0u) |
                   (i + 1 < avail ? static_cast<uint32_t>(d[i + 1]) << 8 : 0u);
        };
        state = word(0) | (word(1) << 16);
        w = 2;
    } else {
        state = J.state0;
    }
    const uint32_t tab_s = static_cast<uint32_t>(__cvta_generic_to_shared(s_tab));
    const uint32_t sym_s = static_cast<uint32_t>(__cvta_generic_to_shared(s_sym));
    const bool slow = (J.flags & kJobSlowRenorm) != 0;
    if (is_se) {
        if (slow) serial_stream<12, true>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, se_sym + J.out_off);
        else serial_stream<12, false>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, se_sym + J.out_off);
    } else {
        if (slow) serial_stream<10, true>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, mant + J.out_off);
        else serial_stream<10, false>(tab_s, sym_s, d, avail, n_words, w, state, J.n_syms, mant + J.out_off);
    }
}

// --------------------------------------------------------------------------
// Segmented un-sort of the legacy formats (one stride-1 stream per tensor).
// --------------------------------------------------------------------------
constexpr int kSegWarps = 8;

// 1. per-segment exponent histograms
__global__ void __launch_bounds__(kSegWarps * 32) seg_hist_kernel(const SegStream *__restrict__ ss,
                                                                  const uint32_t *__restrict__ seg_stream,
                                                                  int n_segs, const uint16_t *__restrict__ se_sym,
                                                                  uint32_t *__restrict__ hist) {
    __shared__ uint32_t h[kSegWarps][256];
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int g = blockIdx.x * kSegWarps + w;
    if (g >= n_segs) return;
    const SegStream S = ss[seg_stream[g]];
    const uint64_t lo = static_cast<uint64_t>(g - S.seg_first) * kSegElems;
    const uint64_t hi = min(S.n, lo + kSegElems);
    for (int e = lane; e < 256; e += 32) h[w][e] = 0;
    __syncwarp();
    const uint16_t *se = se_sym + S.se_off;
    for (uint64_t i = lo + lane; i < hi; i += 32) atomicAdd(&h[w][se[i] & 0xFF], 1u);
    __syncwarp();
    for (int e = lane; e < 256; e += 32) hist[static_cast<uint64_t>(g) * 256 + e] = h[w][e];
}

// 2. one CTA per tensor: totals per exponent, checked against the recorded
//    bucket counts; bucket starts; every segment's cursors (in place)
__global__ void __launch_bounds__(256) seg_scan_kernel(const SegStream *__restrict__ ss,
                                                       const uint2 *__restrict__ buckets,
                                                       uint32_t *__restrict__ hist, uint32_t *errs) {
    __shared__ uint32_t tot[256];
    __shared__ uint32_t s_bad;
    const SegStream S = ss[blockIdx.x];
    const uint32_t e = threadIdx.x;
    uint32_t t = 0;
#pragma unroll 8
    for (uint32_t j = 0; j < S.n_segs; j++) t += hist[static_cast<uint64_t>(S.seg_first + j) * 256 + e];
    tot[e] = t;
    if (e == 0) s_bad = 0;
    __syncthreads();
    for (uint32_t b = e; b < S.n_buckets; b += 256) {
        const uint2 bk = buckets[S.bucket_first + b];
        if (bk.x > 255 || tot[bk.x] != bk.y) s_bad = 1;
    }
    __syncthreads();
    if (s_bad) {
        if (e == 0) atomicOr(&errs[S.tensor], BS_DEV_COUNT);
        return;
    }
    // exclusive scan over exponents (ascending), then over segments
    uint32_t start = 0;
    for (uint32_t k = 0; k < e; k++) start += tot[k];
#pragma unroll 8
    for (uint32_t j = 0; j < S.n_segs; j++) {
        uint32_t *c = &hist[static_cast<uint64_t>(S.seg_first + j) * 256 + e];
        const uint32_t v = *c;
        *c = start;
        start += v;
    }
}

// 3. ranked gather: value i takes the next mantissa of its exponent's bucket
__global__ void __launch_bounds__(kSegWarps * 32) seg_unsort_kernel(
    const SegStream *__restrict__ ss, const uint32_t *__restrict__ seg_stream, int n_segs,
    const uint32_t *__restrict__ hist, const uint16_t *__restrict__ se_sym, const uint8_t *__restrict__ mant,
    const uint32_t *__restrict__ errs) {
    __shared__ uint32_t cur_s[kSegWarps][256];
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int g = blockIdx.x * kSegWarps + w;
    if (g >= n_segs) return;
    const SegStream S = ss[seg_stream[g]];
    if (errs[S.tensor]) return;
    uint32_t *cur = cur_s[w];
    for (int e = lane; e < 256; e += 32) cur[e] = hist[static_cast<uint64_t>(g) * 256 + e];
    __syncwarp();
    const uint64_t lo = static_cast<uint64_t>(g - S.seg_first) * kSegElems;
    const uint64_t hi = min(S.n, lo + kSegElems);
    const uint16_t *se = se_sym + S.se_off;
    const uint8_t *ms = mant + S.mant_off;
    uint16_t *out = reinterpret_cast<uint16_t *>(S.out);
    const uint32_t lt = lanemask_lt_p();
    for (uint64_t i0 = lo; i0 < hi; i0 += 32) {
        const uint64_t i = i0 + lane;
        const bool active = i < hi;
        const uint32_t am = __ballot_sync(kFull, active);
        if (active) {
            const uint32_t s = se[i];
            const uint32_t e = s & 0xFF;
            const uint32_t grp = __match_any_sync(am, e);
            const uint32_t rank = __popc(grp & lt);
            const uint32_t m = ms[cur[e] + rank];
            out[i] = static_cast<uint16_t>((((s >> 8) & 1u) << 15) | (e << 7) | m);
            __syncwarp(am);
            if ((grp & lt) == 0) cur[e] += __popc(grp);
        }
        __syncwarp();
    }
}

cudaError_t launch_seg_merge(const SegStream *d_ss, int n_ss, const uint32_t *d_seg_stream, int n_segs,
                             uint32_t *d_hist, const uint2 *d_buckets, const uint16_t *d_se_sym,
                             const uint8_t *d_mant, uint32_t *d_errs, cudaStream_t s) {
    if (n_ss <= 0 || n_segs <= 0) return cudaSuccess;
    const int blocks = (n_segs + kSegWarps - 1) / kSegWarps;
    seg_hist_kernel<<<blocks, kSegWarps * 32, 0, s>>>(d_ss, d_seg_stream, n_segs, d_se_sym, d_hist);
    seg_scan_kernel<<<n_ss, 256, 0, s>>>(d_ss, d_buckets, d_hist, d_errs);
    seg_unsort_kernel<<<blocks, kSegWarps * 32, 0, s>>>(d_ss, d_seg_stream, n_segs, d_hist, d_se_sym, d_mant,
                                                        d_errs);
    return cudaGetLastError();
}

constexpr int kMergeWarps = 8;

__global__ void __launch_bounds__(kMergeWarps * 32) par_merge_kernel(
    const ParStream *__restrict__ streams, int n_streams_total, const uint2 *__restrict__ buckets,
    const uint16_t *__restrict__ se_sym, const uint8_t *__restrict__ mant, uint32_t *errs) {
    __shared__ uint32_t s_cur[kMergeWarps][256];
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int q = blockIdx.x * kMergeWarps + w;
    if (q >= n_streams_total) return;
    const ParStream S = streams[q];
    uint16_t *out = reinterpret_cast<uint16_t *>(S.out);
    uint32_t *cur = s_cur[w];
    for (int e = lane; e < 256; e += 32) cur[e] = 0;
    __syncwarp();
    const uint16_t *se = se_sym + S.se_off;
    for (uint32_t i = lane; i < S.n_in; i += 32) atomicAdd(&cur[se[i] & 0xFF], 1u);
    __syncwarp();
    // recorded bucket counts must equal the decoded exponent histogram
    uint32_t bad = 0;
    for (uint32_t b = lane; b < S.n_buckets; b += 32) {
        uint2 bk = buckets[S.bucket_first + b];
        if (bk.x > 255 || cur[bk.x] != bk.y) bad = 1;
    }
    bad = __any_sync(kFull, bad);
    if (bad) {
        if (lane == 0) atomicOr(&errs[S.tensor], BS_DEV_COUNT);
        return;
    }
    // exclusive scan of the 256-bin histogram (8 bins per lane)
    uint32_t loc[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        loc[k] = sum;
        sum += cur[lane * 8 + k];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        uint32_t v = __shfl_up_sync(kFull, incl, d);
        if (lane >= static_cast<uint32_t>(d)) incl += v;
    }
    const uint32_t excl = incl - sum;
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; k++) cur[lane * 8 + k] = excl + loc[k];
    __syncwarp();
    const uint32_t lt = lanemask_lt_p();
    const uint8_t *ms = mant + S.mant_off;
    for (uint32_t i0 = 0; i0 < S.n_in; i0 += 32) {
        const uint32_t i = i0 + lane;
        const bool active = i < S.n_in;
        const uint32_t am = __ballot_sync(kFull, active);
        if (active) {
            const uint32_t s = se[i];
            const uint32_t e = s & 0xFF;
            const uint32_t grp = __match_any_sync(am, e);
            const uint32_t rank = __popc(grp & lt);
            const uint32_t m = ms[cur[e] + rank];
            out[S.k + static_cast<uint64_t>(i) * S.stride] =
                static_cast<uint16_t>((((s >> 8) & 1u) << 15) | (e << 7) | m);
            __syncwarp(am);
            if ((grp & lt) == 0) cur[e] += __popc(grp);
        }
        __syncwarp();
    }
}

// Concurrent CTAs of the job kernels on the current device (40 KiB of shared
// memory each).
int par_jobs_slots() {
    int dev = 0, sms = 1, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, par_jobs_kernel, kJobThreads,
                                                      4096 * (sizeof(uint2) + sizeof(uint16_t))) != cudaSuccess)
        cudaGetLastError();
    return sms * (per_sm > 0 ? per_sm : 1);
}

cudaError_t launch_par_jobs(const ParJob *d_jobs, int n_jobs, const uint2 *d_groups, int n_groups,
                            const uint2 *d_tabs, const uint16_t *d_syms, uint16_t *d_se_sym, uint8_t *d_mant,
                            uint32_t *d_errs, cudaStream_t s) {
    // 40 KiB: the larger (SE, 4096-slot) tables; below the 48 KiB default limit
    const size_t smem = 4096 * (sizeof(uint2) + sizeof(uint16_t));
    if (n_groups > 0) {
        par_groups_kernel<<<n_groups, kJobThreads, smem, s>>>(d_jobs, d_groups, d_tabs, d_syms, d_se_sym, d_mant,
                                                              d_errs);
    } else {
        if (n_jobs <= 0) return cudaSuccess;
        par_jobs_kernel<<<n_jobs, kJobThreads, smem, s>>>(d_jobs, d_tabs, d_syms, d_se_sym, d_mant, d_errs);
    }
    return cudaGetLastError();
}

cudaError_t launch_par_merge(const ParStream *d_streams, int n_streams_total, const uint2 *d_buckets,
                             const uint16_t *d_se_sym, const uint8_t *d_mant, uint32_t *d_errs,
                             cudaStream_t s) {
    if (n_streams_total <= 0) return cudaSuccess;
    int blocks = (n_streams_total + kMergeWarps - 1) / kMergeWarps;
    par_merge_kernel<<<blocks, kMergeWarps * 32, 0, s>>>(d_streams, n_streams_total, d_buckets, d_se_sym, d_mant,
                                                         d_errs);
    return cudaGetLastError();
}

}  // namespace bsg
