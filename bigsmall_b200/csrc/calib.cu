// HBM calibration probe (measurement helper for bench.py --config mix; built
// into its own libbscalib.so, not into the product library libbsgpu.so).
//
// A plain grid-stride streaming kernel that reads `rd` and writes `wr` 16-byte
// words per unit with the same access instructions the decoder uses
// (ld.global.nc.L1::no_allocate, st.global.cs).  With rd:wr = 2:3 it moves the
// decoder's read:write byte mix (compressed ~0.66 B read per 2 B written plus
// the plane), so its rate is the practical DRAM ceiling for that mix, next to
// the 1:1 copy figure the roofline denominator is measured with.
#include <cstdint>

#include <cuda_runtime.h>

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

bool on_current_device(const void *p) {
    int dev = 0;
    cudaPointerAttributes a;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeManaged || (a.type == cudaMemoryTypeDevice && a.device == dev);
}

}  // namespace

// `units` x 16-byte words per stream: reads rd streams of d_in and writes wr
// streams of d_out (d_in holds rd*units*16 bytes, d_out wr*units*16),
// grid-stride over `grid` CTAs of 256 threads, on `stream` (a cudaStream_t).
// (rd, wr) in {(1,1), (2,3), (0,1)}.  Returns 0, 1 (bad argument) or 6 (CUDA
// error), the status codes of libbsgpu.so.
extern "C" int bs_stream_probe(const void *d_in, void *d_out, uint64_t units, int rd, int wr, int grid,
                               void *stream) {
    if (!((rd == 1 && wr == 1) || (rd == 2 && wr == 3) || (rd == 0 && wr == 1))) return 1;
    if (grid <= 0 || units == 0 || (rd && !d_in) || !d_out) return 1;
    if ((reinterpret_cast<uintptr_t>(d_in) | reinterpret_cast<uintptr_t>(d_out)) & 15) return 1;
    if ((rd && !on_current_device(d_in)) || !on_current_device(d_out)) return 1;
    auto *in = static_cast<const uint4 *>(d_in);
    auto *out = static_cast<uint4 *>(d_out);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (rd == 1 && wr == 1) stream_mix_kernel<1, 1><<<grid, 256, 0, s>>>(in, out, units);
    else if (rd == 2 && wr == 3) stream_mix_kernel<2, 3><<<grid, 256, 0, s>>>(in, out, units);
    else stream_mix_kernel<0, 1><<<grid, 256, 0, s>>>(in, out, units);
    return cudaGetLastError() == cudaSuccess ? 0 : 6;
}
