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

constexpr int kJobThreads = 128;

// One CTA per serial stream: the CTA stages the stream's decode table
// (slot -> {sym | freq << 16, slot - cum}) in shared memory, then one thread
// runs the stream.  The state stays below 2^32 because the host rejects tables
// with a frequency above M, so 32-bit arithmetic is exact.  The next renorm
// word is loaded as soon as the previous one is consumed, so its latency
// overlaps the following steps' table lookups.
__global__ void __launch_bounds__(kJobThreads) par_jobs_kernel(const ParJob *__restrict__ jobs,
                                                               const uint2 *__restrict__ tabs,
                                                               uint16_t *__restrict__ se_sym,
                                                               uint8_t *__restrict__ mant, uint32_t *errs) {
    extern __shared__ uint2 s_tab[];
    const ParJob J = jobs[blockIdx.x];
    if (J.n_syms == 0) return;
    const bool is_se = (J.flags & kJobSe) != 0;
    const uint32_t prec = is_se ? 12u : 10u;
    const uint32_t M = 1u << prec, mask = M - 1;
    const uint2 *tab = tabs + J.tab_off;
    for (uint32_t i = threadIdx.x; i < M; i += kJobThreads) s_tab[i] = tab[i];
    __syncthreads();
    if (threadIdx.x != 0) return;
    const uint8_t *d = reinterpret_cast<const uint8_t *>(J.data);
    const uint32_t avail = J.avail, n_words = J.n_words;
    auto word = [&](uint32_t k) -> uint32_t {
        const uint32_t i = 2 * k;
        return (i < avail ? static_cast<uint32_t>(d[i]) : 0u) | (i + 1 < avail ? static_cast<uint32_t>(d[i + 1]) << 8 : 0u);
    };
    uint32_t state, w = 0;
    if (J.flags & kJobStateInStream) {
        if (n_words < 2) {   // rans.py:176-177 / numba_rans: a stream shorter than its state
            atomicOr(&errs[J.tensor], BS_DEV_STREAM);
            return;
        }
        state = word(0) | (word(1) << 16);
        w = 2;
    } else {
        state = J.state0;
    }
    uint32_t next = w < n_words ? word(w) : 0u;
    uint16_t *o16 = se_sym + J.out_off;
    uint8_t *o8 = mant + J.out_off;
    for (uint32_t i = 0; i < J.n_syms; i++) {
        const uint2 e = s_tab[state & mask];
        const uint32_t sym = e.x & 0xFFFFu;
        if (is_se) o16[i] = static_cast<uint16_t>(sym);
        else o8[i] = static_cast<uint8_t>(sym);
        state = (e.x >> 16) * (state >> prec) + e.y;
        while (state < kRansL && w < n_words) {
            state = (state << 16) | next;
            w++;
            next = w < n_words ? word(w) : 0u;
        }
    }
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

cudaError_t launch_par_jobs(const ParJob *d_jobs, int n_jobs, const uint2 *d_tabs, uint16_t *d_se_sym,
                            uint8_t *d_mant, uint32_t *d_errs, cudaStream_t s) {
    if (n_jobs <= 0) return cudaSuccess;
    // 32 KiB: the larger (SE, 4096-slot) table; below the 48 KiB default limit
    par_jobs_kernel<<<n_jobs, kJobThreads, 4096 * sizeof(uint2), s>>>(d_jobs, d_tabs, d_se_sym, d_mant, d_errs);
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
