// common.cuh -- shared definitions of the libbsgpu.so kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "bsgpu.h"

namespace bsg {

constexpr uint32_t kRansL = 1u << 16;       // rANS lower bound, 16-bit renorm
constexpr uint32_t kFull = 0xFFFFFFFFu;

// ---- bf16_exp_chunked_v1 layout (little-endian; sections in this order, each
// 16-byte aligned):
//   0 "BSXC" | 4 u16 version (1; 2 with groups) | 6 u8 coder (0 rANS, 1 tANS,
//   2 rANS over exponent pairs) | 7 u8 P
//   8 u64 n | 16 u32 chunk_elems | 20 u32 n_chunks | 24 u32 lanes=32
//   28 u32 aux (coder 2: window base e_lo; else 0)
//   32 u64 chunks_off | 40 u64 plane_off | 48 u64 blob_bytes
//   56 version 1: u64 0; version 2: u32 groups G | u32 0
//   64 u16 freq[256] | 576 u32 group_start[n_groups+1] (16 B units)
//   A chunk is G state groups of ge = chunk_elems / G values (a multiple of
//   256; version 1 is G = 1): group k holds elements [k*ge, min(n, (k+1)*ge)),
//   n_groups = ceil(n / ge), so chunk size (framing) and the number of
//   independently decodable groups (parallelism) are separate choices.
//   plane_off = rup16(576 + 4*(n_groups+1)): n bytes of (sign << 7) | mantissa
//   chunks_off = plane_off + rup16(n): per group [u32 init[32]][u16 words...]
//   zero-padded to 16 B; blob_bytes = end of the last group record.
//   Everything the decode kernels call a "chunk" below is one group.
//   Coder 2 codes the pair (2k, 2k+1) as one symbol a*16 + b, a = e - e_lo
//   for e in [e_lo, e_lo + 14] else 15 (escape; the exponent byte is stored in
//   the record's escape list); its records are [u32 init[32]][u32 n_words]
//   [u32 n_esc][u32 0][u32 0][u16 words][u8 escapes] zero-padded to 16 B.
constexpr uint32_t kXcMagic = 0x43585342u;  // "BSXC" little-endian
constexpr uint32_t kXcFreqOff = 64;
constexpr uint32_t kXcTabOff = 576;
constexpr uint32_t kXcLanes = 32;
constexpr uint32_t kXcMaxTable = 4096;      // 2^12 entries, the largest precision
constexpr uint32_t kXcTableWords = 2 * kXcMaxTable;   // u32 words per tensor's table slot
                                                      // (the pair coder's entries are 8 bytes)
constexpr uint32_t kXcPairRecHdr = 144;     // pair-coder record: 128 B states + 16 B counts

// Device-side tensor descriptor of a decode plan.  The host fills the first
// block; the table-build kernel fills the parsed header fields.  Its "chunks"
// are the blob's state groups (chunk_elems / groups values each).
struct XcTensorDev {
    const uint8_t *blob;
    uint64_t blob_bytes;
    uint16_t *out;
    uint64_t n;
    uint32_t chunk_elems;     // values per group
    uint32_t n_chunks;        // groups in the tensor
    uint32_t chunk_begin;     // first group decoded; d_out holds element chunk_begin * chunk_elems first
    uint32_t aux;             // pair coder: first exponent of the 15-wide window (from the header)
    uint32_t groups;          // groups per chunk in the header (1: format version 1)
    // parsed from the blob header by xc_prepare_kernel
    uint64_t chunks_off;
    uint64_t plane_off;
    uint32_t coder;
    uint32_t prec;
    uint32_t coder_mask;      // from the caller: coders the blob may use (0: any)
    uint32_t rec_lim16;       // end of the chunk-record area in 16-byte units from chunks_off
};

// rANS encode step with the division by the symbol frequency done as a
// multiplication.  The step maps the 32-bit state x (already renormalised, so
// 1 <= x < f * 2^(32-P)) to (x / f) * M + (x mod f) + cum, written as
// x + cum + q * (M - f) with q = floor(x / f).  q = floor(x * m / 2^64) for
// m = ceil(2^64 / f) = floor((2^64 - 1) / f) + 1 (f >= 2): m / 2^64 exceeds
// 1 / f by less than 2^-64, so x * m / 2^64 exceeds x / f by less than 2^-32 <
// 1 / f, which never carries past the next integer.  The 64 x 32 product is two
// 32-bit multiplies, mulhi(x, m_lo) and x * m_hi + that (a 64-bit result whose
// high word is q).  For f = 1, m = 2^64 - 1 gives q = x - 1, and the entry adds
// M - 1 to cum to make up for it.  An entry is {m_lo, m_hi, f << (32 - P)
// (the renorm threshold), cum' | (M - f) << 16}.
__host__ __device__ inline uint4 rans_enc_entry(uint32_t f, uint32_t cum, uint32_t P) {
    const uint32_t M = 1u << P;
    const uint64_t m = f <= 1 ? ~0ull : ~0ull / f + 1;
    const uint32_t fe = f ? f : 1u;
    const uint32_t cw = (cum + (fe == 1 ? M - 1 : 0u)) | ((M - fe) << 16);
    return make_uint4(static_cast<uint32_t>(m), static_cast<uint32_t>(m >> 32), fe << (32 - P), cw);
}

// (x / f) * M + (x mod f) + cum for 1 <= x < f * 2^(32-P), from the entry above
__host__ __device__ inline uint32_t rans_enc_update(uint32_t x, const uint4 &t) {
#ifdef __CUDA_ARCH__
    const uint32_t lo = __umulhi(x, t.x);
#else
    const uint32_t lo = static_cast<uint32_t>((static_cast<uint64_t>(x) * t.x) >> 32);
#endif
    const uint32_t q = static_cast<uint32_t>((static_cast<uint64_t>(x) * t.y + lo) >> 32);
    return x + (t.w & 0xFFFFu) + q * (t.w >> 16);
}

// A work item: up to 16 consecutive chunks of one tensor (xc_warps_per_cta), one CTA.
struct XcItem {
    uint32_t tensor;
    uint32_t first_chunk;
    uint32_t n_chunks;
    uint32_t pad;
};

// ---- bf16_parallel_v1 job descriptors --------------------------------------
// One serial rANS stream (bigsmall/codecs/rans.py:165-207 semantics).
// One serial rANS stream (L = 2^16, 16-bit little-endian renorm words).  The
// three reference readers differ only in where the state comes from and in
// how an odd trailing byte reads; both are folded into (avail, n_words):
// word k = byte 2k | byte 2k+1 << 8 with bytes at or past `avail` reading 0,
// and the decoder may read words [first, n_words).
//   bf16_parallel_v1 (rans.py:165-207): state = words 0,1; an odd last byte is
//     dropped (avail rounded down to even) but still counts as a zero word.
//   bf16_se_tans (numba_rans.py:168-217): state = words 0,1; an odd last byte
//     is the low byte of the last word (avail = the stream length).
//   bf16_se_single_kernel (single_kernel.py:160-190): state stored separately,
//     exactly n_words whole words.
struct ParJob {
    uint64_t data;        // device address of word 0
    uint64_t out_off;     // element offset in the u16 (SE) or u8 (mantissa) scratch
    uint32_t avail;       // stream bytes present (python slices clamp)
    uint32_t n_words;     // words the renorm may read, counting the state words
    uint32_t n_syms;      // symbols to decode
    uint32_t tab_off;     // first entry of its decode table in the plan's table array
    uint32_t state0;      // initial state unless kJobStateInStream
    uint32_t flags;       // kJobSe | kJobStateInStream
    uint32_t tensor;      // index of the plan tensor (its status word)
    uint32_t pad_;
};
constexpr uint32_t kJobSe = 1u;            // u16 (sign,exp) output, P = 12; else u8 mantissa, P = 10
constexpr uint32_t kJobStateInStream = 2u; // state = word 0 | word 1 << 16, renorm from word 2
constexpr uint32_t kJobSlowRenorm = 4u;    // a step may need two renorm words (initial state below
                                           // L, or a table slot with frequency 0)

// Un-sort of one legacy tensor (a single stride-1 stream), split into
// segments of kSegElems values so that every segment's exponent ranks are
// computed by its own warp (histogram, per-exponent scan across segments,
// ranked gather).
constexpr uint32_t kSegElems = 16384;
struct SegStream {
    uint64_t se_off;      // its SE symbols in the u16 scratch
    uint64_t mant_off;    // its sorted mantissas in the u8 scratch
    uint64_t out;         // device address of element 0
    uint64_t n;           // values
    uint32_t seg_first;   // its first segment in the plan's segment list
    uint32_t n_segs;
    uint32_t bucket_first;
    uint32_t n_buckets;
    uint32_t tensor;
    uint32_t pad_;
};

// One stream's merge parameters (a PAR1 stream, or a whole legacy tensor).
struct ParStream {
    uint64_t se_off;      // offset of its SE symbols in the u16 scratch
    uint64_t mant_off;    // offset of its sorted mantissas in the u8 scratch
    uint64_t out;         // device address of element 0 of its tensor's output
    uint32_t n_in;        // elements in the stream
    uint32_t k;           // stream index: its i-th value is element k + i * stride
    uint32_t stride;      // PAR1: the stream count; legacy formats: 1
    uint32_t bucket_first;// index of its first (exponent, count) record
    uint32_t n_buckets;
    uint32_t tensor;      // index of the plan tensor (its status word)
};

}  // namespace bsg

// kernel launchers (host side, defined in the .cu files)
namespace bsg {
cudaError_t launch_xc_prepare(XcTensorDev *d_tens, int n_tensors, uint32_t *d_tables,
                              uint32_t *d_errs, cudaStream_t s);
constexpr uint32_t kXcAllCoders = 7u;   // BS_CODER_RANS | TANS | RANS_PAIR bits
// Union of the tensors' coder masks (a zero mask counts as every coder).
uint32_t xc_launch_mask(const XcTensorDev *h_tens, int n);
cudaError_t launch_xc_decode(const XcTensorDev *d_tens, const XcItem *d_items, int n_items,
                             const uint32_t *d_tables, uint32_t *d_errs, uint32_t coders, int max_ctas,
                             cudaStream_t s);
int xc_warps_per_cta();
cudaError_t xc_decode_attrs(uint32_t coders);   // decode kernels' shared-memory opt-in
cudaError_t launch_xc_noalloc(const XcTensorDev *h_tens, const uint32_t *range_count, int n, cudaStream_t s,
                              uint32_t *h_status);
uint64_t xc_noalloc_scratch_bytes();

// The serial streams: one per CTA (n_groups == 0), or one per warp in groups
// d_groups[g] = {first job, job count <= kJobGroup} of jobs sharing one table.
cudaError_t launch_par_jobs(const ParJob *d_jobs, int n_jobs, const uint2 *d_groups, int n_groups,
                            const uint2 *d_tabs, const uint16_t *d_syms, uint16_t *d_se_sym, uint8_t *d_mant,
                            uint32_t *d_errs, cudaStream_t s);
constexpr uint32_t kJobGroup = 4;   // serial streams per CTA of par_groups_kernel: one per warp
int par_jobs_slots();               // concurrent CTAs of the job kernels on the current device
cudaError_t launch_seg_merge(const SegStream *d_ss, int n_ss, const uint32_t *d_seg_stream, int n_segs,
                             uint32_t *d_hist, const uint2 *d_buckets, const uint16_t *d_se_sym,
                             const uint8_t *d_mant, uint32_t *d_errs, cudaStream_t s);
cudaError_t launch_par_merge(const ParStream *d_streams, int n_streams_total, const uint2 *d_buckets,
                             const uint16_t *d_se_sym, const uint8_t *d_mant, uint32_t *d_errs,
                             cudaStream_t s);

cudaError_t launch_xc_encode(const uint16_t *d_in, uint64_t n, int coder, int prec,
                             uint32_t chunk_elems, uint32_t groups, uint8_t *d_out, uint64_t out_cap,
                             uint64_t *d_out_len, uint8_t *d_ws, uint64_t ws_bytes,
                             cudaStream_t s);
uint64_t xc_encode_workspace(uint64_t n, uint32_t chunk_elems, int coder);
uint64_t xc_encode_bound(uint64_t n, uint32_t chunk_elems);
// (workspace and bound take the values per group; launch_xc_encode codes
// groups of chunk_elems values and writes a header of chunks of
// chunk_elems * groups values)
}  // namespace bsg
