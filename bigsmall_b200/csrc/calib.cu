// HBM calibration probe (measurement helper; not on the decode path).
//
// A plain grid-stride streaming kernel that reads `rd` and writes `wr` 16-byte
// words per unit with the same access instructions the decoder uses
// (ld.global.nc.L1::no_allocate, st.global.cs).  With rd:wr = 2:3 it moves the
// decoder's read:write byte mix (compressed ~0.66 B read per 2 B written plus
// the plane), so its rate is the practical DRAM ceiling for that mix, next to
// the 1:1 copy figure the roofline denominator is measured with.
#include <cstdint>

#include "common.cuh"

namespace bsg {
namespace {

__device__ __forceinline__ uint4 ld_stream16(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream16(uint4 *p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// unit u reads in[u + k*units] (k < RD) and writes out[u + k*units] (k < WR)
template <int RD, int WR>
__global__ void __launch_bounds__(256) stream_mix_kernel(const uint4 *__restrict__ in, uint4 *__restrict__ out,
                                                         uint64_t units) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t u = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; u < units; u += stride) {
        uint4 acc = make_uint4(static_cast<uint32_t>(u), 0, 0, 0);
#pragma unroll
        for (int k = 0; k < RD; k++) {
            const uint4 v = ld_stream16(in + u + k * units);
            acc.x ^= v.x; acc.y ^= v.y; acc.z ^= v.z; acc.w ^= v.w;
        }
#pragma unroll
        for (int k = 0; k < WR; k++) {
            acc.y += k;
            st_stream16(out + u + k * units, acc);
        }
    }
}

}  // namespace

cudaError_t launch_stream_mix(const void *d_in, void *d_out, uint64_t units, int rd, int wr, int grid,
                              cudaStream_t s) {
    auto *in = static_cast<const uint4 *>(d_in);
    auto *out = static_cast<uint4 *>(d_out);
    if (rd == 1 && wr == 1) stream_mix_kernel<1, 1><<<grid, 256, 0, s>>>(in, out, units);
    else if (rd == 2 && wr == 3) stream_mix_kernel<2, 3><<<grid, 256, 0, s>>>(in, out, units);
    else if (rd == 0 && wr == 1) stream_mix_kernel<0, 1><<<grid, 256, 0, s>>>(in, out, units);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace bsg
