/*
 * bsgpu.h -- C ABI of libbsgpu.so, the B200 (sm_100a) decode/encode engine
 * behind BigSmall's bf16 codec path.
 *
 * Plain pointers and sizes only: device pointers are CUDA device addresses,
 * `stream` is a cudaStream_t passed as void*.  Every entry point returns an
 * int status (BS_OK == 0); bs_last_error() gives a message for the calling
 * thread.  Nothing here falls back to the CPU: a device failure is reported,
 * never hidden.
 *
 * Reference interfaces replaced (paths are within the BigSmall project):
 *   bigsmall/kernels/__init__.py:56-64   the missing `ac_cuda` backend slot,
 *                                        contract decode(blob, extras, n)->bytes
 *   bigsmall/kernels/__init__.py:89-111  decode_bf16_parallel dispatch
 *   bigsmall/kernels/ac_triton.py:112-262 Triton SE kernel + CPU mantissa path
 *   bigsmall/codecs/bf16_parallel.py:262-352  bf16_parallel_v1 decode
 *   bigsmall/codecs/kv_cache.py:41-117   KV blob encode/decode (CPU today)
 *   bigsmall/decoder.py:49-97            per-tensor codec dispatch (GPU branch)
 */
#ifndef BSGPU_H
#define BSGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define BS_OK                0
#define BS_E_INVALID_ARG     1   /* bad pointer/size/alignment/parameter      */
#define BS_E_BAD_MAGIC       2   /* blob does not start with its format magic */
#define BS_E_COUNT_MISMATCH  3   /* header n != caller's n_weights            */
#define BS_E_TRUNCATED       4   /* blob shorter than its own framing says    */
#define BS_E_CORRUPT         5   /* device decoder flagged a stream error     */
#define BS_E_CUDA            6   /* a CUDA runtime call failed                */
#define BS_E_UNSUPPORTED     7   /* format version / precision not supported  */
#define BS_E_NOMEM           8   /* allocation failed (plan creation only)    */
#define BS_E_PRECISION       9   /* bf16_parallel_v1 precision mismatch       */

/* per-tensor device status bits (bs_plan_check out array) */
#define BS_DEV_HEADER        0x01u  /* header disagrees with the descriptor   */
#define BS_DEV_FREQ          0x02u  /* frequency table does not sum to 2^P    */
#define BS_DEV_CHUNK_TABLE   0x04u  /* chunk offsets out of range/unordered   */
#define BS_DEV_STREAM        0x08u  /* renorm words over- or under-consumed   */
#define BS_DEV_FINAL_STATE   0x10u  /* coder state did not return to its seed */
#define BS_DEV_COUNT         0x20u  /* bucket/stream symbol counts disagree   */

/* bf16_exp_chunked_v1 coders */
#define BS_CODER_RANS        0
#define BS_CODER_TANS        1
#define BS_CODER_RANS_PAIR   2   /* rANS over exponent pairs (one step per two values) */

typedef struct bs_plan bs_plan;

/* One bf16_exp_chunked_v1 tensor (or a chunk range of one) to decode.  Both
 * pointers must be 16-byte aligned device addresses on the plan's device.
 * chunk_elems and groups come from the container header's per-tensor "extra"
 * dict (bigsmall/container.py:17-38 keeps codec extras there) and must match
 * the blob header.  A chunk is `groups` state groups of chunk_elems / groups
 * values (a multiple of 256), each decoded by its own warp; groups 0 or 1 is a
 * format-version-1 blob (one group per chunk).  Chunks [chunk_begin,
 * chunk_begin + chunk_count) are decoded (chunk_count 0: through the last
 * chunk); d_out receives the value of element chunk_begin * chunk_elems first.
 * Ranges let several GPUs share one tensor. */
typedef struct bs_xc_tensor {
    const void *d_blob;
    uint64_t    blob_bytes;
    void       *d_out;
    uint64_t    n_elems;       /* elements of the whole tensor */
    uint32_t    chunk_elems;
    uint32_t    chunk_begin;
    uint32_t    chunk_count;
    uint32_t    coder_mask;    /* bit c set: the blob may use coder c (BS_CODER_*);
                                  0: any coder.  A plan launches the decode kernel
                                  of each coder its tensors may use; a blob whose
                                  coder is not in a nonzero mask fails with
                                  BS_DEV_HEADER instead of being decoded. */
    uint32_t    groups;        /* state groups per chunk (0 or 1: one) */
    uint32_t    reserved;      /* must be 0 */
} bs_xc_tensor;

/* ---- library ------------------------------------------------------------ */
int         bs_version(void);                 /* 100*major + minor (1.01)    */
const char *bs_last_error(void);              /* thread-local, never NULL    */
const char *bs_status_string(int status);

/* ---- bf16_exp_chunked_v1 decode (the hot path) -------------------------- */
/* Build a reusable decode plan for a batch of tensors (any mix of coders and
 * precisions).  Allocates the plan's device memory (work list, per-tensor
 * decode tables, status words); decoding itself allocates nothing.
 * Replaces: bigsmall/decoder.py:128-136 per-tensor decode loop (GPU branch). */
int bs_xc_plan_create(const bs_xc_tensor *tensors, int n_tensors, int device,
                      bs_plan **out_plan);

/* Enqueue the decode of every tensor in the plan on `stream` (cudaStream_t).
 * Asynchronous; stream-ordered; launches a table-build kernel and the decode
 * kernel.  The plan may be decoded any number of times. */
int bs_plan_decode(bs_plan *plan, void *stream);
/* bs_plan_decode that also records two cudaEvent_t (may be NULL) on the
 * stream right before and right after the decode kernels (after the
 * per-launch table build), so the caller can time the decode kernels alone
 * with cudaEventElapsedTime.  No reference counterpart. */
int bs_plan_decode_timed(bs_plan *plan, void *stream, void *ev_start, void *ev_stop);
/* One call for an event-chained decode on a side stream: the stream waits for
 * `wait_event` (cudaEvent_t, may be NULL), the plan decodes, then `done_event`
 * (may be NULL) is recorded.  Used by the streaming model's per-layer prefetch
 * to keep host work per layer to one call.  For a bf16_exp_chunked_v1 plan the
 * decode's kernels run as one CUDA graph launch (about a quarter of the host
 * time of launching them one by one): the graph is captured on a private
 * stream at the plan's first event-chained call and again after
 * bs_plan_set_max_ctas changes the cap (in relaxed capture mode for the
 * calling thread, so a capture running elsewhere is not disturbed).  When
 * `stream` is itself being captured by the caller, or the graph cannot be
 * captured, the kernels are launched one by one.  No reference counterpart. */
int bs_plan_decode_after(bs_plan *plan, void *stream, void *wait_event, void *done_event);
/* The whole per-layer hand-off of a two-stream prefetch in one call:
 * `release_event` is recorded on `main_stream` (the running layer is done with
 * the slot), `side_stream` waits for it, the plan decodes on `side_stream`,
 * `done_event` is recorded there, and finally `main_stream` waits for
 * `next_event` (the slot of the layer that runs next; may be NULL).  Replaces
 * the reference's prefetch-thread hand-off, bigsmall/streaming_inference.py:
 * 272-348 (decode the next layer while this one runs, swap it in after). */
int bs_plan_decode_handoff(bs_plan *plan, void *main_stream, void *side_stream, void *release_event,
                           void *done_event, void *next_event);

/* Synchronise `stream`, read the per-tensor device status words into
 * `status_out` (may be NULL; else n_tensors entries) and return BS_OK or
 * BS_E_CORRUPT. */
int bs_plan_check(bs_plan *plan, void *stream, uint32_t *status_out);

int bs_plan_n_tensors(const bs_plan *plan);
/* Number of kernels this plan has launched so far (every decode call adds the
 * kernels it enqueued), for measurement.  No reference counterpart. */
int bs_plan_launch_count(const bs_plan *plan, uint64_t *count);
/* Cap the decode grid of a bf16_exp_chunked_v1 plan at max_ctas CTAs (0: one
 * CTA per work item, the default).  A capped plan leaves SM room to kernels on
 * other streams, e.g. a layer decode overlapped with the previous layer's
 * GEMMs; the CTAs walk the work list until it is done.  No reference
 * counterpart. */
int bs_plan_set_max_ctas(bs_plan *plan, int max_ctas);
int bs_plan_destroy(bs_plan *plan);

/* ---- allocation-free decode -------------------------------------------- */
/* No counterpart in the reference.  Decodes up to BS_NOALLOC_MAX_TENSORS
 * bf16_exp_chunked_v1 tensors (descriptors as for bs_xc_plan_create) on
 * `stream` without allocating any device memory: for callers that cannot call
 * cudaMalloc -- e.g. a serving engine that has already reserved nearly all of
 * HBM for its own arena or KV cache (a fresh cudaMalloc can fail there), or a
 * latency-critical path where cudaMalloc/cudaFree would synchronise the whole
 * device.  Its scratch (descriptors, decode tables, status words; about
 * 260 KiB) is a static device array that every GPU loading the library holds
 * until the process exits.  The first call on a device resolves that array's
 * address (with the device current); make that first call before any stream
 * capture.  With CUDA's lazy module loading (the default in CUDA 12) the
 * library's kernels and this array are loaded into a device's context on
 * first use, which itself needs a little device memory: make one call (or set
 * CUDA_MODULE_LOADING=EAGER) before the caller reserves its HBM.  The resolved
 * address belongs to the device's current context; after cudaDeviceReset the
 * process must not call this entry point again on that device.  All calls
 * share the array, so calls whose GPU work overlaps race: serialise them.
 * Synchronous: returns after `stream` has finished the decode, with the
 * per-tensor device status words in `status_out` (may be NULL; else n_tensors
 * entries).  More than BS_NOALLOC_MAX_TENSORS tensors is BS_E_INVALID_ARG. */
#define BS_NOALLOC_MAX_TENSORS 8
int bs_xc_decode_noalloc(const bs_xc_tensor *tensors, int n_tensors, void *stream,
                         uint32_t *status_out);

/* ---- bf16_parallel_v1 decode (the reference's GPU format) --------------- */
/* Parse a PAR1 blob's framing on the host (`h_blob`, the same bytes as at
 * `d_blob` on the device) and build a decode plan writing n_weights bf16
 * values to d_out.  Errors mirror bigsmall/codecs/bf16_parallel.py:153-163,
 * :274-276 (bad magic, precision mismatch, count mismatch).
 * Replaces: bigsmall/kernels/ac_triton.py:112-262 and
 *           bigsmall/codecs/bf16_parallel.py:262-352. */
int bs_par_plan_create(const uint8_t *h_blob, uint64_t blob_bytes,
                       uint64_t n_weights, const void *d_blob, void *d_out,
                       int device, bs_plan **out_plan);

/* ---- legacy serial formats (bf16_se_single_kernel, bf16_se_tans) --------- */
/* One serial (sign,exp) rANS stream per tensor plus one rANS stream per
 * exponent bucket of mantissas, un-sorted by exponent: the device runs every
 * stream of the tensor concurrently (one CTA each) and then the un-sort, so a
 * tensor decodes in the time of its (sign,exp) stream.  Same plan object and
 * calls as bf16_parallel_v1 (bs_plan_decode / bs_plan_check / bs_plan_destroy).
 * Replaces: bigsmall/codecs/single_kernel.py:432-613 (decode) and
 *           bigsmall/codecs/bf16_tans.py:121-167 + numba_rans.py:168-217. */
#define BS_SE_SINGLE_KERNEL 1
#define BS_SE_TANS          2
/* bf16_parallel_v1 blobs in a bs_se_plan_create_many batch: their N slice
 * streams join the batch's concurrent streams (one bs_par_plan_create per
 * tensor runs its tensors one after another). */
#define BS_SE_PARALLEL      3
int bs_se_plan_create(int codec, const uint8_t *h_blob, uint64_t blob_bytes,
                      uint64_t n_weights, const void *d_blob, void *d_out,
                      int device, bs_plan **out_plan);
/* Many legacy tensors in one plan: all their serial streams run concurrently,
 * so a batch decodes in the time of its longest (sign,exp) stream; one status
 * word per blob.  `h_blob` holds the same bytes as `d_blob`. */
typedef struct bs_se_blob {
    int            codec;        /* BS_SE_SINGLE_KERNEL, BS_SE_TANS or BS_SE_PARALLEL */
    const uint8_t *h_blob;
    uint64_t       blob_bytes;
    uint64_t       n_weights;
    const void    *d_blob;
    void          *d_out;        /* n_weights bf16 values */
} bs_se_blob;
int bs_se_plan_create_many(const bs_se_blob *blobs, int n_blobs, int device, bs_plan **out_plan);
/* Host-only framing check of a legacy blob (no device work): BS_OK and the
 * number of serial streams, or the status bs_se_plan_create would return. */
int bs_se_parse(int codec, const uint8_t *h_blob, uint64_t blob_bytes,
                uint64_t n_weights, uint32_t *n_streams_out);

/* ---- bf16_exp_chunked_v1 encode (KV-cache compression) ------------------ */
/* Worst-case blob size, and scratch size for one tensor with a given coder,
 * for chunks of chunk_elems values in `groups` state groups (0 or 1: one). */
int bs_xc_encode_bound(uint64_t n_elems, uint32_t chunk_elems, uint32_t groups, uint64_t *bytes);
int bs_xc_encode_workspace(uint64_t n_elems, uint32_t chunk_elems, uint32_t groups, int coder,
                           uint64_t *bytes);

/* Encode n_elems bf16 values at d_in into a bf16_exp_chunked_v1 blob at d_out
 * (capacity out_cap >= bs_xc_encode_bound).  Chunks of chunk_elems values are
 * cut into `groups` state groups (chunk_elems / groups must be a multiple of
 * 256; groups > 1 writes format version 2).  The exact blob length is written
 * to the device u64 at d_out_len.  Deterministic: the bytes equal the CPU
 * reference encoder's.  Coder 2 quantises a product of its two window-index
 * marginals, counted over every value, or for n_elems >= 2^20 over the
 * 2048-value blocks whose index is a multiple of 8; coders 0 and 1 count every
 * value.  Asynchronous on `stream`: one memset and five kernels, so a run of
 * encodes can be captured into a CUDA graph (relaxed capture mode; the KV
 * benchmark replays a whole step of 64 encodes that way).
 * Replaces: bigsmall/codecs/kv_cache.py:41-83 compress_kv_entry's CPU encode. */
int bs_xc_encode(const void *d_in, uint64_t n_elems, int coder, int prec,
                 uint32_t chunk_elems, uint32_t groups, void *d_out, uint64_t out_cap,
                 uint64_t *d_out_len, void *d_workspace, uint64_t ws_bytes,
                 void *stream);

#ifdef __cplusplus
}
#endif
#endif /* BSGPU_H */
