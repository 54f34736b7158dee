// par_decode.cu -- sm_100a decoder of the reference's bf16_parallel_v1 format.
//
// The reference decodes this format with one Triton program per stream for the
// (sign,exp) substream only, then decodes every mantissa bucket, un-sorts and
// merges on the CPU (bigsmall/kernels/ac_triton.py:172-262).  Here everything
// stays on the device:
//   par_jobs_kernel   one thread per serial rANS stream: every stream's SE
//                     substream and every (stream, exponent) mantissa bucket is
//                     an independent job, all decoded concurrently with the
//                     exact bigsmall/codecs/rans.py:165-207 state machine
//                     (including its end-of-data zero fill).
//   par_merge_kernel  one warp per stream: rebuilds the stream's bucket starts
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

__global__ void __launch_bounds__(128) par_jobs_kernel(const uint8_t *__restrict__ blob,
                                                       const ParJob *__restrict__ jobs, int n_jobs,
                                                       const uint2 *__restrict__ se_tab,
                                                       const uint2 *__restrict__ m_tabs,
                                                       uint16_t *__restrict__ se_sym,
                                                       uint8_t *__restrict__ mant, uint32_t *err) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n_jobs) return;
    const ParJob J = jobs[j];
    if (J.n_syms == 0) return;
    const uint8_t *d = blob + J.data_off;
    const uint32_t len = J.data_len;
    if (len < 4) {           // rans.py:176-177 raises on a blob shorter than its state
        atomicOr(err, BS_DEV_STREAM);
        return;
    }
    const uint32_t prec = J.is_se ? 12u : 10u;
    const uint32_t mask = (1u << prec) - 1;
    const uint2 *tab = J.is_se ? se_tab : m_tabs + static_cast<uint64_t>(J.table - 1) * 1024;
    uint64_t state = static_cast<uint64_t>(d[0]) | (static_cast<uint64_t>(d[1]) << 8) |
                     (static_cast<uint64_t>(d[2]) << 16) | (static_cast<uint64_t>(d[3]) << 24);
    uint32_t pos = 4;
    for (uint32_t i = 0; i < J.n_syms; i++) {
        const uint32_t slot = static_cast<uint32_t>(state) & mask;
        const uint2 e = tab[slot];
        const uint32_t sym = e.x & 0xFFFF;
        if (J.is_se) se_sym[J.out_off + i] = static_cast<uint16_t>(sym);
        else mant[J.out_off + i] = static_cast<uint8_t>(sym);
        state = static_cast<uint64_t>(e.x >> 16) * (state >> prec) + slot - e.y;
        while (state < kRansL && pos < len) {
            if (pos + 2 > len) {       // one byte left: shift in zeros and stop
                state <<= 16;
                pos = len;
                break;
            }
            state = (state << 16) | d[pos] | (static_cast<uint32_t>(d[pos + 1]) << 8);
            pos += 2;
        }
    }
}

constexpr int kMergeWarps = 8;

__global__ void __launch_bounds__(kMergeWarps * 32) par_merge_kernel(
    const ParStream *__restrict__ streams, int n_streams_total, const uint2 *__restrict__ buckets,
    const uint16_t *__restrict__ se_sym, const uint8_t *__restrict__ mant, uint16_t *__restrict__ out,
    uint32_t n_streams, uint32_t *err) {
    __shared__ uint32_t s_cur[kMergeWarps][256];
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int q = blockIdx.x * kMergeWarps + w;
    if (q >= n_streams_total) return;
    const ParStream S = streams[q];
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
        if (lane == 0) atomicOr(err, BS_DEV_COUNT);
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
            out[S.k + static_cast<uint64_t>(i) * n_streams] =
                static_cast<uint16_t>((((s >> 8) & 1u) << 15) | (e << 7) | m);
            __syncwarp(am);
            if ((grp & lt) == 0) cur[e] += __popc(grp);
        }
        __syncwarp();
    }
}

cudaError_t launch_par_jobs(const uint8_t *d_blob, const ParJob *d_jobs, int n_jobs, const uint2 *d_se_tab,
                            const uint2 *d_m_tabs, uint16_t *d_se_sym, uint8_t *d_mant, uint32_t *d_err,
                            cudaStream_t s) {
    if (n_jobs <= 0) return cudaSuccess;
    par_jobs_kernel<<<(n_jobs + 127) / 128, 128, 0, s>>>(d_blob, d_jobs, n_jobs, d_se_tab, d_m_tabs, d_se_sym,
                                                         d_mant, d_err);
    return cudaGetLastError();
}

cudaError_t launch_par_merge(const ParStream *d_streams, int n_streams_total, const uint32_t *d_buckets,
                             const uint16_t *d_se_sym, const uint8_t *d_mant, uint16_t *d_out,
                             uint32_t n_streams, uint32_t *d_err, cudaStream_t s) {
    if (n_streams_total <= 0) return cudaSuccess;
    int blocks = (n_streams_total + kMergeWarps - 1) / kMergeWarps;
    par_merge_kernel<<<blocks, kMergeWarps * 32, 0, s>>>(d_streams, n_streams_total,
                                                         reinterpret_cast<const uint2 *>(d_buckets), d_se_sym,
                                                         d_mant, d_out, n_streams, d_err);
    return cudaGetLastError();
}

}  // namespace bsg
