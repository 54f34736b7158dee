// capi.cu -- the C ABI of libbsgpu.so (declared in include/bsgpu.h).
//
// Host-side responsibilities: argument validation (pointer residency and
// alignment are checked before any kernel can touch them), plan construction
// (work lists, bf16_parallel_v1 framing parse), kernel launches, and turning
// device status words into status codes.  No entry point falls back to a CPU
// decoder.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

using namespace bsg;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}
int cuda_fail(cudaError_t e, const char *what) {
    g_err = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return BS_E_CUDA;
}

struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) {
            changed = cudaSetDevice(dev) == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

// The pointer must be device (or managed) memory of `device`; anything else
// would make a kernel fault, so it is rejected here.
bool on_device(const void *p, int device) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeManaged) return true;
    return a.type == cudaMemoryTypeDevice && a.device == device;
}

inline uint64_t rup(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

// little-endian readers for host-side PAR1 parsing
inline uint32_t rd16(const uint8_t *p) { return p[0] | (p[1] << 8); }
inline uint32_t rd32(const uint8_t *p) {
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
           (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
}

}  // namespace

enum PlanKind { kPlanXc = 1, kPlanPar = 2 };

struct bs_plan {
    int kind = 0;
    int device = 0;
    int n_tensors = 0;          // as given by the caller
    void *d_mem = nullptr;
    uint32_t *d_errs = nullptr; // one word per internal tensor
    uint32_t *h_errs = nullptr; // pinned mirror
    int n_internal = 0;
    std::vector<int> user_to_internal;   // -1: empty tensor, nothing to decode
    // bf16_exp_chunked_v1
    XcTensorDev *d_tens = nullptr;
    XcItem *d_items = nullptr;
    int n_items = 0;
    uint32_t coders = 0;        // decode kernels to launch (bit per coder)
    int max_ctas = 0;           // decode grid cap (0: one CTA per work item)
    uint32_t *d_tables = nullptr;
    // serial-stream formats (bf16_parallel_v1, bf16_se_single_kernel, bf16_se_tans)
    ParJob *d_jobs = nullptr;
    int n_jobs = 0;
    uint2 *d_groups = nullptr;   // {first job, job count}: jobs sharing a decode table
    int n_groups = 0;
    ParStream *d_streams = nullptr;
    int n_streams_total = 0;
    uint2 *d_buckets = nullptr;
    uint2 *d_tabs = nullptr;
    uint16_t *d_syms = nullptr;
    uint16_t *d_se_sym = nullptr;
    uint8_t *d_mant = nullptr;
    SegStream *d_ss = nullptr;      // legacy tensors: segmented un-sort
    int n_ss = 0;
    uint32_t *d_seg_stream = nullptr;
    int n_segs = 0;
    uint32_t *d_hist = nullptr;
    uint64_t launches = 0;          // kernels this plan has launched (bs_plan_launch_count)
    // bf16_exp_chunked_v1: the table build + decode kernels as one CUDA graph,
    // captured on first use by the event-chained calls (decode_after, handoff)
    cudaGraphExec_t graph = nullptr;
    int graph_ctas = -1;            // max_ctas the graph was captured with
    bool graph_failed = false;      // capture not possible here: plain launches from then on
};

namespace {

// carve a single device allocation into aligned sub-buffers
struct Carve {
    uint64_t off = 0;
    uint64_t take(uint64_t bytes, uint64_t align = 256) {
        off = rup(off, align);
        uint64_t r = off;
        off += bytes;
        return r;
    }
};

int alloc_plan_mem(bs_plan *p, uint64_t bytes) {
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc(&p->d_mem, bytes);
    if (e != cudaSuccess) {
        p->d_mem = nullptr;
        cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? fail(BS_E_NOMEM, "cudaMalloc of plan memory failed")
                                              : cuda_fail(e, "cudaMalloc");
    }
    return BS_OK;
}

void free_plan(bs_plan *p) {
    if (!p) return;
    DeviceGuard g(p->device);
    if (p->graph) cudaGraphExecDestroy(p->graph);
    if (p->d_mem) cudaFree(p->d_mem);
    if (p->h_errs) cudaFreeHost(p->h_errs);
    delete p;
}

// Validate one bf16_exp_chunked_v1 descriptor and turn it into the device
// descriptor of its state groups: the decode kernels work per group, so the
// chunk range [chunk_begin, chunk_begin + chunk_count) becomes the group range
// [*g_begin, *g_begin + *g_count).  `who` prefixes error messages.
int xc_describe(const bs_xc_tensor &t, int device, const std::string &who, XcTensorDev *d, uint32_t *g_begin,
                uint32_t *g_count) {
    if (t.coder_mask & ~kXcAllCoders) return fail(BS_E_INVALID_ARG, who + "coder_mask has unknown coder bits");
    if (t.reserved) return fail(BS_E_INVALID_ARG, who + "reserved field must be 0");
    if (!t.d_blob || !t.d_out) return fail(BS_E_INVALID_ARG, who + "NULL pointer");
    if ((reinterpret_cast<uintptr_t>(t.d_blob) | reinterpret_cast<uintptr_t>(t.d_out)) & 15)
        return fail(BS_E_INVALID_ARG, who + "blob and output must be 16-byte aligned");
    const uint32_t G = t.groups ? t.groups : 1u;
    if (t.chunk_elems == 0 || t.chunk_elems % G || (t.chunk_elems / G) < 256 || ((t.chunk_elems / G) & 255))
        return fail(BS_E_INVALID_ARG, who + "chunk_elems / groups must be a positive multiple of 256");
    const uint32_t ge = t.chunk_elems / G;
    const uint64_t nc = (t.n_elems + t.chunk_elems - 1) / t.chunk_elems;
    const uint64_t ng = (t.n_elems + ge - 1) / ge;
    if (ng > 0x7FFFFFFFull) return fail(BS_E_INVALID_ARG, who + "too many chunks");
    if (t.chunk_begin >= nc) return fail(BS_E_INVALID_ARG, who + "chunk_begin beyond the last chunk");
    const uint64_t cnt = t.chunk_count ? t.chunk_count : nc - t.chunk_begin;
    if (t.chunk_begin + cnt > nc) return fail(BS_E_INVALID_ARG, who + "chunk range beyond the last chunk");
    const uint64_t min_bytes = rup(kXcTabOff + 4 * (ng + 1), 16) + rup(t.n_elems, 16) + 128 * ng;
    if (t.blob_bytes < min_bytes) return fail(BS_E_TRUNCATED, who + "blob shorter than its framing");
    if (!on_device(t.d_blob, device) || !on_device(t.d_out, device))
        return fail(BS_E_INVALID_ARG, who + "pointers must be device memory of device " + std::to_string(device));
    const uint64_t gb = static_cast<uint64_t>(t.chunk_begin) * G;
    const uint64_t ge_end = std::min<uint64_t>(ng, (t.chunk_begin + cnt) * G);
    XcTensorDev x{};
    x.blob = static_cast<const uint8_t *>(t.d_blob);
    x.blob_bytes = t.blob_bytes;
    x.out = static_cast<uint16_t *>(t.d_out);
    x.n = t.n_elems;
    x.chunk_elems = ge;
    x.n_chunks = static_cast<uint32_t>(ng);
    x.chunk_begin = static_cast<uint32_t>(gb);
    x.aux = 0;
    x.groups = G;
    x.coder = 0xFFFFFFFFu;
    x.coder_mask = t.coder_mask;
    *d = x;
    *g_begin = static_cast<uint32_t>(gb);
    *g_count = static_cast<uint32_t>(ge_end - gb);
    return BS_OK;
}

}  // namespace

extern "C" {

int bs_version(void) { return 101; }

const char *bs_last_error(void) { return g_err.c_str(); }

const char *bs_status_string(int status) {
    switch (status) {
        case BS_OK: return "ok";
        case BS_E_INVALID_ARG: return "invalid argument";
        case BS_E_BAD_MAGIC: return "bad magic";
        case BS_E_COUNT_MISMATCH: return "weight count mismatch";
        case BS_E_TRUNCATED: return "truncated blob";
        case BS_E_CORRUPT: return "corrupt stream";
        case BS_E_CUDA: return "CUDA error";
        case BS_E_UNSUPPORTED: return "unsupported format";
        case BS_E_NOMEM: return "out of device memory";
        case BS_E_PRECISION: return "precision mismatch";
        default: return "unknown status";
    }
}

int bs_plan_set_max_ctas(bs_plan *p, int max_ctas) {
    if (!p) return fail(BS_E_INVALID_ARG, "plan is NULL");
    if (max_ctas < 0) return fail(BS_E_INVALID_ARG, "max_ctas must be >= 0");
    if (p->kind != kPlanXc) return fail(BS_E_INVALID_ARG, "max_ctas applies to bf16_exp_chunked_v1 plans");
    p->max_ctas = max_ctas;
    return BS_OK;
}

int bs_plan_n_tensors(const bs_plan *plan) { return plan ? plan->n_tensors : 0; }

int bs_plan_launch_count(const bs_plan *plan, uint64_t *count) {
    if (!plan || !count) return fail(BS_E_INVALID_ARG, "plan or count is NULL");
    *count = plan->launches;
    return BS_OK;
}

int bs_plan_destroy(bs_plan *plan) {
    free_plan(plan);
    return BS_OK;
}

// --------------------------------------------------------------------------
// bf16_exp_chunked_v1
// --------------------------------------------------------------------------
int bs_xc_plan_create(const bs_xc_tensor *tensors, int n_tensors, int device, bs_plan **out_plan) {
    if (!out_plan) return fail(BS_E_INVALID_ARG, "out_plan is NULL");
    *out_plan = nullptr;
    if (n_tensors < 0 || (n_tensors > 0 && !tensors)) return fail(BS_E_INVALID_ARG, "bad tensor array");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return fail(BS_E_INVALID_ARG, "invalid CUDA device " + std::to_string(device));
    }
    DeviceGuard guard(device);
    std::vector<XcTensorDev> ht;
    std::vector<std::pair<uint32_t, uint32_t>> ranges;   // chunk range per internal tensor
    std::vector<int> u2i(n_tensors, -1);
    for (int i = 0; i < n_tensors; i++) {
        const bs_xc_tensor &t = tensors[i];
        if (t.n_elems == 0) continue;
        XcTensorDev d;
        uint32_t gb = 0, gc = 0;
        const int rc = xc_describe(t, device, "tensor " + std::to_string(i) + ": ", &d, &gb, &gc);
        if (rc) return rc;
        u2i[i] = static_cast<int>(ht.size());
        ht.push_back(d);
        ranges.push_back({gb, gc});
    }
    // work items: <= warps-per-CTA chunks of one tensor; big tensors first so
    // small ones fill the tail of the grid
    const uint32_t W = static_cast<uint32_t>(xc_warps_per_cta());
    std::vector<int> order(ht.size());
    for (size_t i = 0; i < ht.size(); i++) order[i] = static_cast<int>(i);
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return ranges[a].second > ranges[b].second; });
    std::vector<XcItem> items;
    for (int ti : order) {
        const uint32_t c0 = ranges[ti].first, c1 = ranges[ti].first + ranges[ti].second;
        for (uint32_t c = c0; c < c1; c += W) {
            XcItem it{static_cast<uint32_t>(ti), c, std::min(W, c1 - c), 0};
            items.push_back(it);
        }
    }
    if (items.size() > 0x7FFFFFFFull) return fail(BS_E_INVALID_ARG, "too many work items");
    auto *p = new bs_plan();
    p->kind = kPlanXc;
    p->device = device;
    p->n_tensors = n_tensors;
    p->n_internal = static_cast<int>(ht.size());
    p->user_to_internal = u2i;
    p->n_items = static_cast<int>(items.size());
    p->coders = xc_launch_mask(ht.data(), static_cast<int>(ht.size()));
    Carve cv;
    const uint64_t o_t = cv.take(sizeof(XcTensorDev) * ht.size());
    const uint64_t o_i = cv.take(sizeof(XcItem) * items.size());
    const uint64_t o_e = cv.take(4 * ht.size());
    const uint64_t o_tab = cv.take(4ull * kXcTableWords * ht.size());
    int rc = alloc_plan_mem(p, cv.off);
    if (rc) { free_plan(p); return rc; }
    auto *base = static_cast<uint8_t *>(p->d_mem);
    p->d_tens = reinterpret_cast<XcTensorDev *>(base + o_t);
    p->d_items = reinterpret_cast<XcItem *>(base + o_i);
    p->d_errs = reinterpret_cast<uint32_t *>(base + o_e);
    p->d_tables = reinterpret_cast<uint32_t *>(base + o_tab);
    cudaError_t e = cudaSuccess;
    if (!ht.empty()) e = cudaMemcpy(p->d_tens, ht.data(), sizeof(XcTensorDev) * ht.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !items.empty())
        e = cudaMemcpy(p->d_items, items.data(), sizeof(XcItem) * items.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !ht.empty()) e = cudaMemset(p->d_errs, 0, 4 * ht.size());
    if (e == cudaSuccess) e = cudaMallocHost(&p->h_errs, 4 * std::max<size_t>(1, ht.size()));
    if (e != cudaSuccess) {
        rc = cuda_fail(e, "plan upload");
        free_plan(p);
        return rc;
    }
    *out_plan = p;
    return BS_OK;
}

// Kernels one decode of a bf16_exp_chunked_v1 plan launches: the table build
// plus one decode kernel per coder family the plan may meet.
static uint64_t xc_kernels_per_decode(const bs_plan *p) {
    if (p->n_items <= 0) return 1;
    return 1 + ((p->coders & ((1u << BS_CODER_RANS) | (1u << BS_CODER_TANS))) ? 1 : 0) +
           ((p->coders & (1u << BS_CODER_RANS_PAIR)) ? 1 : 0);
}

// The decode step of a plan; `ev_start` / `ev_stop` (cudaEvent_t, optional)
// are recorded on the stream right before and after the decode kernels, after
// the table build, so a caller can time the decode kernels alone.
static int plan_decode(bs_plan *p, void *stream, void *ev_start, void *ev_stop) {
    if (!p) return fail(BS_E_INVALID_ARG, "plan is NULL");
    DeviceGuard guard(p->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    auto mark = [&](void *ev) {
        if (ev && e == cudaSuccess) e = cudaEventRecord(static_cast<cudaEvent_t>(ev), s);
    };
    if (p->kind == kPlanXc) {
        if (p->n_internal == 0) { mark(ev_start); mark(ev_stop); return e == cudaSuccess ? BS_OK : cuda_fail(e, "event"); }
        e = launch_xc_prepare(p->d_tens, p->n_internal, p->d_tables, p->d_errs, s);
        mark(ev_start);
        if (e == cudaSuccess)
            e = launch_xc_decode(p->d_tens, p->d_items, p->n_items, p->d_tables, p->d_errs, p->coders,
                                 p->max_ctas, s);
        if (e == cudaSuccess) p->launches += xc_kernels_per_decode(p);
        mark(ev_stop);
    } else if (p->kind == kPlanPar) {
        mark(ev_start);
        if (p->n_internal > 0) {
            if (e == cudaSuccess) e = cudaMemsetAsync(p->d_errs, 0, 4ull * p->n_internal, s);
            if (e == cudaSuccess) {
                e = launch_par_jobs(p->d_jobs, p->n_jobs, p->d_groups, p->n_groups, p->d_tabs, p->d_syms,
                                    p->d_se_sym, p->d_mant, p->d_errs, s);
                if (e == cudaSuccess && (p->n_groups > 0 || p->n_jobs > 0)) p->launches += 1;
            }
            if (e == cudaSuccess) {
                e = launch_par_merge(p->d_streams, p->n_streams_total, p->d_buckets, p->d_se_sym, p->d_mant,
                                     p->d_errs, s);
                if (e == cudaSuccess && p->n_streams_total > 0) p->launches += 1;
            }
            if (e == cudaSuccess) {
                e = launch_seg_merge(p->d_ss, p->n_ss, p->d_seg_stream, p->n_segs, p->d_hist, p->d_buckets,
                                     p->d_se_sym, p->d_mant, p->d_errs, s);
                if (e == cudaSuccess && p->n_ss > 0 && p->n_segs > 0) p->launches += 3;
            }
        }
        mark(ev_stop);
    } else {
        return fail(BS_E_INVALID_ARG, "unknown plan kind");
    }
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    return BS_OK;
}

int bs_plan_decode(bs_plan *p, void *stream) { return plan_decode(p, stream, nullptr, nullptr); }

// Kernels of one bf16_exp_chunked_v1 decode as a single graph launch: about a
// quarter of the host time of launching them one by one, which matters to a
// per-layer prefetch beside a host-bound model.  The graph is captured on a
// private stream (thread-local capture mode) the first time, and again after
// the plan's CTA cap changes; it refers only to the plan's own memory.
static int plan_decode_graph(bs_plan *p, cudaStream_t s) {
    if (p->kind != kPlanXc || p->n_internal == 0 || p->graph_failed) return plan_decode(p, s, nullptr, nullptr);
    DeviceGuard guard(p->device);
    // a caller capturing `s` records the kernels themselves into its graph
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return plan_decode(p, s, nullptr, nullptr);
    }
    cudaError_t e = cudaSuccess;
    if (!p->graph || p->graph_ctas != p->max_ctas) {
        if (p->graph) {
            cudaGraphExecDestroy(p->graph);
            p->graph = nullptr;
        }
        // relaxed mode for this thread: creating the private stream must not
        // invalidate a global-mode capture running elsewhere in the process
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        e = xc_decode_attrs(p->coders);
        cudaStream_t cs = nullptr;
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (e == cudaSuccess) {
            cudaError_t le = launch_xc_prepare(p->d_tens, p->n_internal, p->d_tables, p->d_errs, cs);
            if (le == cudaSuccess)
                le = launch_xc_decode(p->d_tens, p->d_items, p->n_items, p->d_tables, p->d_errs, p->coders,
                                      p->max_ctas, cs);
            cudaGraph_t g = nullptr;
            e = cudaStreamEndCapture(cs, &g);
            if (e == cudaSuccess) e = le;
            if (e == cudaSuccess) e = cudaGraphInstantiate(&p->graph, g, 0);
            if (g) cudaGraphDestroy(g);
        }
        if (cs) cudaStreamDestroy(cs);
        cudaThreadExchangeStreamCaptureMode(&mode);   // the caller's mode back
        if (e != cudaSuccess) {
            // e.g. the calling thread is inside a global-mode stream capture:
            // the same kernels are launched one by one instead
            if (p->graph) cudaGraphExecDestroy(p->graph);
            p->graph = nullptr;
            p->graph_failed = true;
            cudaGetLastError();
            return plan_decode(p, s, nullptr, nullptr);
        }
        p->graph_ctas = p->max_ctas;
    }
    e = cudaGraphLaunch(p->graph, s);
    if (e != cudaSuccess) return cuda_fail(e, "decode graph launch");
    p->launches += xc_kernels_per_decode(p);
    return BS_OK;
}

int bs_plan_decode_timed(bs_plan *p, void *stream, void *ev_start, void *ev_stop) {
    return plan_decode(p, stream, ev_start, ev_stop);
}

int bs_plan_decode_after(bs_plan *p, void *stream, void *wait_event, void *done_event) {
    if (!p) return fail(BS_E_INVALID_ARG, "plan is NULL");
    DeviceGuard guard(p->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (wait_event) {
        const cudaError_t e = cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(wait_event), 0);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
    }
    const int rc = plan_decode_graph(p, s);
    if (rc) return rc;
    if (done_event) {
        const cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(done_event), s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    }
    return BS_OK;
}

int bs_plan_decode_handoff(bs_plan *p, void *main_stream, void *side_stream, void *release_event,
                           void *done_event, void *next_event) {
    if (!p) return fail(BS_E_INVALID_ARG, "plan is NULL");
    if (!release_event || !done_event) return fail(BS_E_INVALID_ARG, "hand-off needs release and done events");
    DeviceGuard guard(p->device);
    cudaStream_t m = static_cast<cudaStream_t>(main_stream);
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(release_event), m);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(release)");
    const int rc = bs_plan_decode_after(p, side_stream, release_event, done_event);
    if (rc) return rc;
    if (next_event) {
        e = cudaStreamWaitEvent(m, static_cast<cudaEvent_t>(next_event), 0);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent(next)");
    }
    return BS_OK;
}

int bs_plan_check(bs_plan *p, void *stream, uint32_t *status_out) {
    if (!p) return fail(BS_E_INVALID_ARG, "plan is NULL");
    DeviceGuard guard(p->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (p->n_internal > 0)
        e = cudaMemcpyAsync(p->h_errs, p->d_errs, 4ull * p->n_internal, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "status readback");
    bool bad = false;
    std::string msg;
    for (int i = 0; i < p->n_tensors; i++) {
        int k = p->user_to_internal[i];
        uint32_t st = k >= 0 ? p->h_errs[k] : 0u;
        if (status_out) status_out[i] = st;
        if (st) {
            if (!bad) msg = "tensor " + std::to_string(i) + " device status 0x" + [&] {
                char b[16];
                snprintf(b, sizeof b, "%x", st);
                return std::string(b);
            }();
            bad = true;
        }
    }
    if (bad) return fail(BS_E_CORRUPT, msg);
    return BS_OK;
}

// --------------------------------------------------------------------------
// allocation-free decode: same validation as bs_xc_plan_create, scratch in a
// static device array (xc_decode.cu), no cudaMalloc/cudaFree anywhere
// --------------------------------------------------------------------------
int bs_xc_decode_noalloc(const bs_xc_tensor *tensors, int n_tensors, void *stream, uint32_t *status_out) {
    if (n_tensors < 0 || n_tensors > BS_NOALLOC_MAX_TENSORS)
        return fail(BS_E_INVALID_ARG, "bs_xc_decode_noalloc decodes at most " +
                                          std::to_string(BS_NOALLOC_MAX_TENSORS) + " tensors per call (got " +
                                          std::to_string(n_tensors) + ")");
    if (n_tensors > 0 && !tensors) return fail(BS_E_INVALID_ARG, "tensors is NULL");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return fail(BS_E_CUDA, "no current CUDA device");
    }
    XcTensorDev ht[BS_NOALLOC_MAX_TENSORS];
    uint32_t rc_count[BS_NOALLOC_MAX_TENSORS];
    int u2i[BS_NOALLOC_MAX_TENSORS];
    int n = 0;
    for (int i = 0; i < n_tensors; i++) {
        const bs_xc_tensor &t = tensors[i];
        u2i[i] = -1;
        if (t.n_elems == 0) continue;
        uint32_t gb = 0, gc = 0;
        const int rc = xc_describe(t, device, "tensor " + std::to_string(i) + ": ", &ht[n], &gb, &gc);
        if (rc) return rc;
        rc_count[n] = gc;
        u2i[i] = n++;
    }
    uint32_t st[BS_NOALLOC_MAX_TENSORS] = {};
    if (n > 0) {
        cudaError_t e = launch_xc_noalloc(ht, rc_count, n, static_cast<cudaStream_t>(stream), st);
        if (e != cudaSuccess) return cuda_fail(e, "bs_xc_decode_noalloc");
    }
    bool bad = false;
    std::string msg;
    for (int i = 0; i < n_tensors; i++) {
        const uint32_t w = u2i[i] >= 0 ? st[u2i[i]] : 0u;
        if (status_out) status_out[i] = w;
        if (w && !bad) {
            char b[16];
            snprintf(b, sizeof b, "%x", w);
            msg = "tensor " + std::to_string(i) + " device status 0x" + b;
            bad = true;
        }
    }
    if (bad) return fail(BS_E_CORRUPT, msg);
    return BS_OK;
}

// --------------------------------------------------------------------------
// bf16_parallel_v1 (bigsmall/codecs/bf16_parallel.py:15-52 layout)
// --------------------------------------------------------------------------
}  // extern "C"

// --------------------------------------------------------------------------
// Serial-stream formats: bf16_parallel_v1 and the legacy bf16_se_* codecs.
// The host parses the framing into independent rANS jobs (one per SE stream
// and per exponent bucket), per-stream merge records and decode tables; the
// device runs par_jobs_kernel + par_merge_kernel.
// --------------------------------------------------------------------------
namespace {

struct SerialLayout {
    std::vector<ParJob> jobs;
    std::vector<ParStream> streams;      // PAR1 streams (warp-per-stream un-sort)
    std::vector<SegStream> segs;         // legacy tensors (segmented un-sort)
    std::vector<uint32_t> seg_stream;    // per segment: index into segs
    std::vector<uint2> buckets;          // (exponent, count) per stream, blob order
    std::vector<uint2> tabs;             // decode tables {freq, slot - cum}: 4096 (SE) or 1024 entries each
    std::vector<uint16_t> syms;          // slot -> symbol, same indexing as tabs
    uint64_t n_total = 0;                // values of all tensors (scratch size)
};

// Bounds-checked little-endian reader over the host copy of a blob.  `take`
// clamps like a Python slice / BytesIO.read; the others fail on truncation.
struct Rd {
    const uint8_t *h;
    uint64_t len, pos;
    bool bad = false;
    bool need(uint64_t k) {
        if (bad || pos + k > len || pos + k < pos) { bad = true; return false; }
        return true;
    }
    uint32_t u8() { if (!need(1)) return 0; return h[pos++]; }
    uint32_t u16() { if (!need(2)) return 0; uint32_t v = rd16(h + pos); pos += 2; return v; }
    uint32_t u32() { if (!need(4)) return 0; uint32_t v = rd32(h + pos); pos += 4; return v; }
    uint64_t take(uint64_t k, uint64_t *got) {
        const uint64_t at = pos, avail = pos < len ? len - pos : 0;
        *got = std::min(k, avail);
        pos += *got;
        return at;
    }
};

// Append a decode table: slot -> {freq[sym], slot - cum[sym]} and slot -> sym;
// slots past the frequency sum map to symbol 0 (rans.build_slot_to_symbol /
// numba_rans zero-initialised tables).  Frequencies above M are rejected,
// which keeps the decoder's 32-bit state exact.  Returns the table's first
// entry, or -1; *zero_slot tells whether some slot has frequency 0 (its step
// can need a second renorm word).
int64_t add_table(SerialLayout &L, const std::vector<uint32_t> &f, uint32_t M, bool *zero_slot = nullptr) {
    std::vector<uint32_t> cum(f.size());
    uint64_t c = 0;
    for (size_t s = 0; s < f.size(); s++) {
        if (f[s] > M) return -1;
        cum[s] = static_cast<uint32_t>(std::min<uint64_t>(c, 0xFFFFFFFFull));
        c += f[s];
    }
    const size_t base = L.tabs.size();
    if (base + M > 0xFFFFFFFFull) return -1;
    L.tabs.resize(base + M);
    L.syms.resize(base + M);
    for (uint32_t slot = 0; slot < M; slot++) {
        L.tabs[base + slot] = make_uint2(f[0], slot);
        L.syms[base + slot] = 0;
    }
    for (size_t s = 0; s < f.size(); s++)
        for (uint64_t j = 0; j < f[s] && cum[s] + j < M; j++) {
            L.tabs[base + cum[s] + j] = make_uint2(f[s], static_cast<uint32_t>(j));
            L.syms[base + cum[s] + j] = static_cast<uint16_t>(s);
        }
    if (zero_slot) *zero_slot = c < M && f[0] == 0;
    return static_cast<int64_t>(base);
}

// state a stream-state job starts from (word 0 | word 1 << 16, bytes past
// `avail` read as zero)
uint32_t stream_state(const uint8_t *h, uint64_t avail) {
    uint32_t v = 0;
    for (uint64_t i = 0; i < 4; i++) v |= (i < avail ? static_cast<uint32_t>(h[i]) : 0u) << (8 * i);
    return v;
}

// mark jobs whose steps can need two renorm words (kJobSlowRenorm)
void mark_slow(ParJob &j, const uint8_t *h_job, bool zero_slot) {
    const uint32_t st = (j.flags & kJobStateInStream) ? stream_state(h_job, j.avail) : j.state0;
    if (zero_slot || st < kRansL) j.flags |= kJobSlowRenorm;
}

uint64_t freq_sum(const std::vector<uint32_t> &f) {
    uint64_t c = 0;
    for (uint32_t v : f) c += v;
    return c;
}

ParJob word_job(uint64_t addr, uint64_t avail, uint64_t n_words, uint64_t n_syms, uint32_t tab_off, uint32_t flags,
                uint32_t tensor, uint32_t state0 = 0) {
    ParJob j{};
    j.data = addr;
    j.out_off = 0;
    j.avail = static_cast<uint32_t>(avail);
    j.n_words = static_cast<uint32_t>(n_words);
    j.n_syms = static_cast<uint32_t>(n_syms);
    j.tab_off = tab_off;
    j.state0 = state0;
    j.flags = flags;
    j.tensor = tensor;
    return j;
}

// rans.py stream of `got` bytes: state = bytes 0..3, words from byte 4, an odd
// last byte dropped (shifted in as a zero word)
ParJob rans_py_job(uint64_t addr, uint64_t got, uint64_t n_syms, uint32_t tab_off, uint32_t flags, uint32_t tensor) {
    const uint64_t avail = got < 4 ? got : 4 + ((got - 4) & ~1ull);
    const uint64_t n_words = got < 4 ? got / 2 : 2 + (got - 4 + 1) / 2;
    return word_job(addr, avail, n_words, n_syms, tab_off, flags | kJobStateInStream, tensor);
}

// numba_rans stream of `got` bytes: zero-padded to even length, read as u16
ParJob numba_job(uint64_t addr, uint64_t got, uint64_t n_syms, uint32_t tab_off, uint32_t flags, uint32_t tensor) {
    return word_job(addr, got, (got + 1) / 2, n_syms, tab_off, flags | kJobStateInStream, tensor);
}

// One blob being added to a layout: host bytes, device address, output.
struct SerialBlob {
    const uint8_t *h;
    uint64_t len;
    uint64_t n_weights;
    uint64_t d_blob;       // device address of byte 0 (0 while only parsing)
    uint64_t d_out;
    uint32_t tensor;
};

// Finish one stream: bucket jobs get their offset in the stream's sorted
// mantissa run (buckets in ascending exponent order, rans bincount/cumsum).
int finish_stream(SerialLayout &L, ParStream S, std::vector<std::pair<uint32_t, ParJob>> &bj, const std::string &who) {
    std::vector<uint64_t> cnt(256, 0);
    uint64_t total = 0;
    for (auto &x : bj) { cnt[x.first] = x.second.n_syms; total += x.second.n_syms; }
    if (total != S.n_in) return fail(BS_E_CORRUPT, who + "bucket counts do not sum to the value count");
    std::vector<uint64_t> bstart(257, 0);
    for (int e = 0; e < 256; e++) bstart[e + 1] = bstart[e] + cnt[e];
    for (auto &x : bj) {
        x.second.out_off = S.mant_off + bstart[x.first];
        L.jobs.push_back(x.second);
    }
    L.streams.push_back(S);
    return BS_OK;
}

// _unpack_header + decode, bigsmall/codecs/bf16_parallel.py:138-183, :262-352
int parse_par1(SerialLayout &L, const SerialBlob &B) {
    const uint8_t *h = B.h;
    const uint64_t len = B.len;
    Rd r{h, len, 0};
    const char *T = "bf16_parallel: blob truncated in header";
    if (len < 4) return fail(BS_E_TRUNCATED, T);
    if (memcmp(h, "PAR1", 4) != 0) return fail(BS_E_BAD_MAGIC, "bf16_parallel: bad magic");
    r.pos = 4;
    const uint64_t n = r.u32();
    const uint32_t ns = r.u16(), p_se = r.u16(), p_m = r.u16();
    if (r.bad) return fail(BS_E_TRUNCATED, T);
    if (p_se != 12 || p_m != 10)
        return fail(BS_E_PRECISION, "bf16_parallel: precision mismatch (header SE=" + std::to_string(p_se) +
                                        " M=" + std::to_string(p_m) + " vs codec SE=12 M=10)");
    const uint32_t n_se_nz = r.u16();
    if (!r.need(6ull * n_se_nz)) return fail(BS_E_TRUNCATED, T);
    std::vector<uint32_t> se_f(512, 0);
    for (uint32_t i = 0; i < n_se_nz; i++) {
        const uint32_t s = rd16(h + r.pos + 2 * i);
        if (s >= 512) return fail(BS_E_CORRUPT, "bf16_parallel: SE symbol index out of range");
        se_f[s] = rd32(h + r.pos + 2ull * n_se_nz + 4 * i);
    }
    r.pos += 6ull * n_se_nz;
    const uint32_t n_exps = r.u32();
    if (!r.need(2ull * n_exps)) return fail(BS_E_TRUNCATED, T);
    const uint64_t exps_pos = r.pos;
    r.pos += 2ull * n_exps;
    std::vector<int> exp_tab(256, -1);
    std::vector<std::vector<uint32_t>> mfreq;
    for (uint32_t q = 0; q < n_exps; q++) {
        const uint32_t ev = rd16(h + exps_pos + 2 * q);
        const uint32_t nzc = r.u8();
        if (!r.need(5ull * nzc)) return fail(BS_E_TRUNCATED, T);
        if (ev >= 256) return fail(BS_E_CORRUPT, "bf16_parallel: exponent out of range");
        std::vector<uint32_t> mf(128, 0);
        for (uint32_t i = 0; i < nzc; i++) {
            const uint32_t m = h[r.pos + i];
            if (m >= 128) return fail(BS_E_CORRUPT, "bf16_parallel: mantissa index out of range");
            mf[m] = rd32(h + r.pos + nzc + 4 * i);
        }
        r.pos += 5ull * nzc;
        if (exp_tab[ev] < 0) {
            exp_tab[ev] = static_cast<int>(mfreq.size());
            mfreq.push_back(mf);
        } else {
            mfreq[exp_tab[ev]] = mf;   // later entries overwrite (dict semantics)
        }
    }
    if (n != B.n_weights)
        return fail(BS_E_COUNT_MISMATCH, "bf16_parallel: weight count mismatch (" + std::to_string(n) + " vs " +
                                             std::to_string(B.n_weights) + ")");
    if (ns == 0) return fail(BS_E_CORRUPT, "bf16_parallel: zero streams");
    const uint64_t n_off = static_cast<uint64_t>(ns) + 1;
    if (!r.need(4 * n_off)) return fail(BS_E_TRUNCATED, "bf16_parallel: offset table truncated");
    const uint8_t *offt = h + r.pos;
    const uint64_t payload_start = r.pos + 4 * n_off;
    bool se_zero = false;
    const int64_t se_tab = add_table(L, se_f, 4096, &se_zero);
    if (se_tab < 0) return fail(BS_E_CORRUPT, "bf16_parallel: SE frequency above M");
    std::vector<uint32_t> m_tab(mfreq.size());
    std::vector<uint8_t> m_zero(mfreq.size());
    for (size_t t = 0; t < mfreq.size(); t++) {
        bool z = false;
        const int64_t o = add_table(L, mfreq[t], 1024, &z);
        if (o < 0) return fail(BS_E_CORRUPT, "bf16_parallel: mantissa frequency above M");
        m_tab[t] = static_cast<uint32_t>(o);
        m_zero[t] = z;
    }
    uint64_t se_cur = L.n_total;
    for (uint32_t k = 0; k < ns; k++) {
        const uint64_t nin = k < n ? (n - 1 - k) / ns + 1 : 0;
        if (nin == 0) continue;
        uint64_t a = payload_start + rd32(offt + 4ull * k), b = payload_start + rd32(offt + 4ull * (k + 1));
        a = std::min(a, len);
        b = std::min(b, len);
        if (b < a) b = a;
        Rd s{h, b, a};
        const std::string who = "bf16_parallel: stream " + std::to_string(k) + ": ";
        const uint32_t se_len = s.u32();
        if (s.bad) return fail(BS_E_TRUNCATED, who + "truncated");
        uint64_t got;
        const uint64_t se_at = s.take(se_len, &got);
        L.jobs.push_back(rans_py_job(B.d_blob + se_at, got, nin, static_cast<uint32_t>(se_tab), kJobSe, B.tensor));
        L.jobs.back().out_off = se_cur;
        mark_slow(L.jobs.back(), h + se_at, se_zero);
        const uint32_t nze = s.u32();
        if (!s.need(2ull * nze)) return fail(BS_E_TRUNCATED, who + "truncated");
        const uint64_t sx = s.pos;
        s.pos += 2ull * nze;
        ParStream S{};
        S.se_off = se_cur;
        S.mant_off = se_cur;
        S.out = B.d_out;
        S.n_in = static_cast<uint32_t>(nin);
        S.k = k;
        S.stride = ns;
        S.bucket_first = static_cast<uint32_t>(L.buckets.size());
        S.n_buckets = nze;
        S.tensor = B.tensor;
        std::vector<uint8_t> seen(256, 0);
        std::vector<std::pair<uint32_t, ParJob>> bj;
        for (uint32_t qq = 0; qq < nze; qq++) {
            const uint32_t ev = rd16(h + sx + 2ull * qq);
            const uint32_t count = s.u32(), blen = s.u32();
            if (s.bad) return fail(BS_E_TRUNCATED, who + "truncated");
            const uint64_t at = s.take(blen, &got);
            if (ev >= 256 || exp_tab[ev] < 0) return fail(BS_E_CORRUPT, who + "bucket exponent has no table");
            if (seen[ev]) return fail(BS_E_CORRUPT, who + "duplicate bucket exponent");
            seen[ev] = 1;
            bj.push_back({ev, rans_py_job(B.d_blob + at, got, count, m_tab[exp_tab[ev]], 0, B.tensor)});
            mark_slow(bj.back().second, h + at, m_zero[exp_tab[ev]]);
            L.buckets.push_back(make_uint2(ev, count));
        }
        const int rc = finish_stream(L, S, bj, who);
        if (rc) return rc;
        se_cur += nin;
    }
    L.n_total += n;
    return BS_OK;
}

// One legacy tensor: SE job + bucket jobs, contiguous output, segmented
// un-sort.  Bucket jobs land at their exponent's start in the tensor's sorted
// mantissa run (ascending exponents, rans bincount/cumsum).
int finish_legacy(SerialLayout &L, const SerialBlob &B, uint64_t n, uint32_t bucket_first,
                  std::vector<std::pair<uint32_t, ParJob>> &bj, const std::string &who) {
    std::vector<uint64_t> cnt(256, 0);
    uint64_t total = 0;
    for (auto &x : bj) { cnt[x.first] = x.second.n_syms; total += x.second.n_syms; }
    if (total != n) return fail(BS_E_CORRUPT, who + "bucket counts do not sum to the value count");
    std::vector<uint64_t> bstart(257, 0);
    for (int e = 0; e < 256; e++) bstart[e + 1] = bstart[e] + cnt[e];
    for (auto &x : bj) {
        x.second.out_off = L.n_total + bstart[x.first];
        L.jobs.push_back(x.second);
    }
    SegStream S{};
    S.se_off = L.n_total;
    S.mant_off = L.n_total;
    S.out = B.d_out;
    S.n = n;
    S.seg_first = static_cast<uint32_t>(L.seg_stream.size());
    S.n_segs = static_cast<uint32_t>((n + kSegElems - 1) / kSegElems);
    S.bucket_first = bucket_first;
    S.n_buckets = static_cast<uint32_t>(L.buckets.size()) - bucket_first;
    S.tensor = B.tensor;
    for (uint32_t j = 0; j < S.n_segs; j++) L.seg_stream.push_back(static_cast<uint32_t>(L.segs.size()));
    L.segs.push_back(S);
    L.n_total += n;
    return BS_OK;
}

// bigsmall/codecs/single_kernel.py:432-580 _decode_full_kernel framing:
// [u32 n][u16 n_se_nz][u16 sym x n_se_nz][u32 freq x n_se_nz][u32 state][u32 n_words][u16 x n_words]
// [u32 n_buckets] then per bucket [u16 e][u8 mnz][u8 sym x mnz][u32 freq x mnz][u32 state][u32 count]
// [u32 n_words][u16 x n_words].  Tables must sum to M (the reference would
// leave slots uninitialised otherwise).
int parse_sk(SerialLayout &L, const SerialBlob &B) {
    const uint8_t *h = B.h;
    Rd r{h, B.len, 0};
    const char *T = "bf16_se_single_kernel: blob truncated";
    const uint64_t n = r.u32();
    if (r.bad) return fail(BS_E_TRUNCATED, T);
    if (n != B.n_weights)
        return fail(BS_E_COUNT_MISMATCH, "bf16_se_single_kernel: weight count mismatch (" + std::to_string(n) +
                                             " vs " + std::to_string(B.n_weights) + ")");
    const uint32_t n_se_nz = r.u16();
    if (!r.need(6ull * n_se_nz)) return fail(BS_E_TRUNCATED, T);
    std::vector<uint32_t> se_f(512, 0);
    for (uint32_t i = 0; i < n_se_nz; i++) {
        const uint32_t s = rd16(h + r.pos + 2 * i);
        if (s >= 512) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: SE symbol out of range");
        se_f[s] = rd32(h + r.pos + 2ull * n_se_nz + 4 * i);
    }
    r.pos += 6ull * n_se_nz;
    if (freq_sum(se_f) != 4096) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: SE frequencies do not sum to 4096");
    bool se_zero = false;
    const int64_t se_tab = add_table(L, se_f, 4096, &se_zero);
    if (se_tab < 0) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: SE frequency above M");
    const uint32_t st = r.u32(), nc = r.u32();
    if (!r.need(2ull * nc)) return fail(BS_E_TRUNCATED, T);
    ParJob se = word_job(B.d_blob + r.pos, 2ull * nc, nc, n, static_cast<uint32_t>(se_tab), kJobSe, B.tensor, st);
    se.out_off = L.n_total;
    mark_slow(se, h + r.pos, se_zero);
    L.jobs.push_back(se);
    r.pos += 2ull * nc;
    const uint32_t nb = r.u32();
    if (r.bad) return fail(BS_E_TRUNCATED, T);
    const uint32_t bucket_first = static_cast<uint32_t>(L.buckets.size());
    std::vector<uint8_t> seen(256, 0);
    std::vector<std::pair<uint32_t, ParJob>> bj;
    for (uint32_t q = 0; q < nb; q++) {
        const uint32_t e = r.u16(), mnz = r.u8();
        if (!r.need(5ull * mnz)) return fail(BS_E_TRUNCATED, T);
        if (e >= 256) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: exponent out of range");
        std::vector<uint32_t> mf(128, 0);
        for (uint32_t i = 0; i < mnz; i++) {
            const uint32_t m = h[r.pos + i];
            if (m >= 128) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: mantissa symbol out of range");
            mf[m] = rd32(h + r.pos + mnz + 4 * i);
        }
        r.pos += 5ull * mnz;
        if (freq_sum(mf) != 1024) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: mantissa frequencies do not sum to 1024");
        const uint32_t mst = r.u32(), bsize = r.u32(), mnc = r.u32();
        if (!r.need(2ull * mnc)) return fail(BS_E_TRUNCATED, T);
        if (seen[e]) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: duplicate bucket exponent");
        seen[e] = 1;
        bool z = false;
        const int64_t t = add_table(L, mf, 1024, &z);
        if (t < 0) return fail(BS_E_CORRUPT, "bf16_se_single_kernel: mantissa frequency above M");
        bj.push_back({e, word_job(B.d_blob + r.pos, 2ull * mnc, mnc, bsize, static_cast<uint32_t>(t), 0, B.tensor, mst)});
        mark_slow(bj.back().second, h + r.pos, z);
        L.buckets.push_back(make_uint2(e, bsize));
        r.pos += 2ull * mnc;
    }
    return finish_legacy(L, B, n, bucket_first, bj, "bf16_se_single_kernel: ");
}

// bigsmall/codecs/bf16_tans.py:121-167 framing (streams are numba_rans.py
// rANS streams, :168-217): [u32 n][u16 se_nz][u16 sym x se_nz][u32 freq x se_nz]
// [u32 cw_len][SE stream][u32 m_len][m section]; m section = [u32 n_exps]
// [u16 e x n_exps] then per exponent [u32 count][u8 nnz][u8 sym x nnz]
// [u32 freq x nnz][u32 len][stream].  Payload reads clamp like BytesIO.read.
int parse_setans(SerialLayout &L, const SerialBlob &B) {
    const uint8_t *h = B.h;
    Rd r{h, B.len, 0};
    const char *T = "bf16_se_tans: blob truncated";
    const uint64_t n = r.u32();
    if (r.bad) return fail(BS_E_TRUNCATED, T);
    if (n != B.n_weights)
        return fail(BS_E_COUNT_MISMATCH, "bf16_se_tans: weight count mismatch (" + std::to_string(n) + " vs " +
                                             std::to_string(B.n_weights) + ")");
    const uint32_t se_nz = r.u16();
    if (!r.need(6ull * se_nz)) return fail(BS_E_TRUNCATED, T);
    std::vector<uint32_t> se_f(512, 0);
    for (uint32_t i = 0; i < se_nz; i++) {
        const uint32_t s = rd16(h + r.pos + 2 * i);
        if (s >= 512) return fail(BS_E_CORRUPT, "bf16_se_tans: SE symbol out of range");
        se_f[s] = rd32(h + r.pos + 2ull * se_nz + 4 * i);
    }
    r.pos += 6ull * se_nz;
    const uint32_t cwl = r.u32();
    if (r.bad) return fail(BS_E_TRUNCATED, T);
    uint64_t got;
    const uint64_t cw = r.take(cwl, &got);
    if (got < 4) return fail(BS_E_TRUNCATED, "bf16_se_tans: SE stream shorter than its state");
    bool se_zero = false;
    const int64_t se_tab = add_table(L, se_f, 4096, &se_zero);
    if (se_tab < 0) return fail(BS_E_CORRUPT, "bf16_se_tans: SE frequency above M");
    ParJob se = numba_job(B.d_blob + cw, got, n, static_cast<uint32_t>(se_tab), kJobSe, B.tensor);
    se.out_off = L.n_total;
    mark_slow(se, h + cw, se_zero);
    L.jobs.push_back(se);
    const uint32_t mbl = r.u32();
    if (r.bad) return fail(BS_E_TRUNCATED, T);
    const uint64_t mb = r.take(mbl, &got);
    Rd m{h, mb + got, mb};
    const uint32_t ne = m.u32();
    if (!m.need(2ull * ne)) return fail(BS_E_TRUNCATED, T);
    const uint64_t ex = m.pos;
    m.pos += 2ull * ne;
    const uint32_t bucket_first = static_cast<uint32_t>(L.buckets.size());
    std::vector<uint8_t> seen(256, 0);
    std::vector<std::pair<uint32_t, ParJob>> bj;
    for (uint32_t q = 0; q < ne; q++) {
        const uint32_t ev = rd16(h + ex + 2ull * q);
        const uint32_t nb = m.u32(), nnz = m.u8();
        if (!m.need(5ull * nnz)) return fail(BS_E_TRUNCATED, T);
        std::vector<uint32_t> mf(128, 0);
        bool bad_sym = false;
        for (uint32_t i = 0; i < nnz; i++) {
            const uint32_t s = h[m.pos + i];
            if (s >= 128) bad_sym = true;
            else mf[s] = rd32(h + m.pos + nnz + 4 * i);
        }
        m.pos += 5ull * nnz;
        const uint32_t cl = m.u32();
        if (m.bad) return fail(BS_E_TRUNCATED, T);
        uint64_t cgot;
        const uint64_t c2 = m.take(cl, &cgot);
        if (ev >= 256 || bad_sym) return fail(BS_E_CORRUPT, "bf16_se_tans: bucket symbol out of range");
        if (seen[ev]) return fail(BS_E_CORRUPT, "bf16_se_tans: duplicate bucket exponent");
        seen[ev] = 1;
        if (nb > 0 && cgot < 4) return fail(BS_E_TRUNCATED, "bf16_se_tans: bucket stream shorter than its state");
        bool z = false;
        const int64_t t = add_table(L, mf, 1024, &z);
        if (t < 0) return fail(BS_E_CORRUPT, "bf16_se_tans: mantissa frequency above M");
        bj.push_back({ev, numba_job(B.d_blob + c2, cgot, nb, static_cast<uint32_t>(t), 0, B.tensor)});
        mark_slow(bj.back().second, h + c2, z);
        L.buckets.push_back(make_uint2(ev, nb));
    }
    return finish_legacy(L, B, n, bucket_first, bj, "bf16_se_tans: ");
}

int parse_serial(int codec, SerialLayout &L, const SerialBlob &B) {
    switch (codec) {
        case BS_SE_SINGLE_KERNEL: return parse_sk(L, B);
        case BS_SE_TANS: return parse_setans(L, B);
        case BS_SE_PARALLEL: return parse_par1(L, B);
        default: return fail(BS_E_INVALID_ARG, "unknown legacy codec " + std::to_string(codec));
    }
}

// Upload a parsed layout into a new plan (kind kPlanPar) over n_tensors user
// tensors; u2i maps them to status words (-1: nothing to decode).
int make_serial_plan(SerialLayout &L, int device, int n_tensors, std::vector<int> u2i, int n_internal,
                     bs_plan **out_plan) {
    // Two schedules for the serial streams.  One stream per CTA (longest
    // first) runs each chain fastest but holds a 40 KiB table per stream, so
    // at most par_jobs_slots() run at once; streams sharing a table (the
    // slices of a bf16_parallel_v1 tensor) can instead run one per warp,
    // kJobGroup per CTA, at a per-chain cost measured 16 % higher.  Pick the
    // smaller estimated makespan: max(longest stream, symbols in flight / slots).
    std::stable_sort(L.jobs.begin(), L.jobs.end(), [](const ParJob &x, const ParJob &y) {
        return x.tab_off != y.tab_off ? x.tab_off < y.tab_off : x.n_syms > y.n_syms;
    });
    std::vector<uint2> groups;
    double longest = 0, total = 0, group_total = 0;
    for (size_t i = 0; i < L.jobs.size(); i++) {
        if (groups.empty() || L.jobs[i].tab_off != L.jobs[groups.back().x].tab_off || groups.back().y == kJobGroup) {
            groups.push_back(make_uint2(static_cast<uint32_t>(i), 0));
            group_total += L.jobs[i].n_syms;   // a group holds its CTA for its longest stream
        }
        groups.back().y++;
        longest = std::max(longest, static_cast<double>(L.jobs[i].n_syms));
        total += L.jobs[i].n_syms;
    }
    const double slots = L.jobs.empty() ? 1.0 : static_cast<double>(par_jobs_slots());
    const double t_single = std::max(longest, total / slots);
    const double t_grouped = 1.16 * std::max(longest, group_total / slots);
    if (groups.size() < L.jobs.size() && t_grouped < t_single) {
        std::stable_sort(groups.begin(), groups.end(), [&](const uint2 &a, const uint2 &b) {
            return L.jobs[a.x].n_syms > L.jobs[b.x].n_syms;
        });
    } else {
        groups.clear();
        std::stable_sort(L.jobs.begin(), L.jobs.end(),
                         [](const ParJob &x, const ParJob &y) { return x.n_syms > y.n_syms; });
    }
    if (L.jobs.size() > 0x7FFFFFFFull || L.streams.size() > 0x7FFFFFFFull || L.seg_stream.size() > 0x7FFFFFFFull)
        return fail(BS_E_INVALID_ARG, "too many streams");
    auto *p = new bs_plan();
    p->kind = kPlanPar;
    p->device = device;
    p->n_tensors = n_tensors;
    p->user_to_internal = std::move(u2i);
    p->n_internal = n_internal;
    if (n_internal == 0) {
        *out_plan = p;
        return BS_OK;
    }
    Carve cv;
    const uint64_t o_j = cv.take(sizeof(ParJob) * L.jobs.size());
    const uint64_t o_g = cv.take(sizeof(uint2) * groups.size());
    const uint64_t o_s = cv.take(sizeof(ParStream) * L.streams.size());
    const uint64_t o_b = cv.take(sizeof(uint2) * std::max<size_t>(1, L.buckets.size()));
    const uint64_t o_t = cv.take(sizeof(uint2) * std::max<size_t>(1, L.tabs.size()));
    const uint64_t o_sy = cv.take(sizeof(uint16_t) * std::max<size_t>(1, L.syms.size()));
    const uint64_t o_sg = cv.take(sizeof(SegStream) * L.segs.size());
    const uint64_t o_sgs = cv.take(sizeof(uint32_t) * L.seg_stream.size());
    const uint64_t o_h = cv.take(256ull * sizeof(uint32_t) * L.seg_stream.size());
    const uint64_t o_ss = cv.take(2 * L.n_total);
    const uint64_t o_m = cv.take(L.n_total);
    const uint64_t o_e = cv.take(4ull * n_internal);
    int rc = alloc_plan_mem(p, cv.off);
    if (rc) { free_plan(p); return rc; }
    auto *base = static_cast<uint8_t *>(p->d_mem);
    p->d_jobs = reinterpret_cast<ParJob *>(base + o_j);
    p->n_jobs = static_cast<int>(L.jobs.size());
    p->d_groups = reinterpret_cast<uint2 *>(base + o_g);
    p->n_groups = static_cast<int>(groups.size());
    p->d_streams = reinterpret_cast<ParStream *>(base + o_s);
    p->n_streams_total = static_cast<int>(L.streams.size());
    p->d_buckets = reinterpret_cast<uint2 *>(base + o_b);
    p->d_tabs = reinterpret_cast<uint2 *>(base + o_t);
    p->d_syms = reinterpret_cast<uint16_t *>(base + o_sy);
    p->d_ss = reinterpret_cast<SegStream *>(base + o_sg);
    p->n_ss = static_cast<int>(L.segs.size());
    p->d_seg_stream = reinterpret_cast<uint32_t *>(base + o_sgs);
    p->n_segs = static_cast<int>(L.seg_stream.size());
    p->d_hist = reinterpret_cast<uint32_t *>(base + o_h);
    p->d_se_sym = reinterpret_cast<uint16_t *>(base + o_ss);
    p->d_mant = base + o_m;
    p->d_errs = reinterpret_cast<uint32_t *>(base + o_e);
    cudaError_t e = cudaSuccess;
    auto up = [&](void *dst, const void *src, size_t bytes) {
        if (e == cudaSuccess && bytes) e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    };
    up(p->d_jobs, L.jobs.data(), sizeof(ParJob) * L.jobs.size());
    up(p->d_groups, groups.data(), sizeof(uint2) * groups.size());
    up(p->d_streams, L.streams.data(), sizeof(ParStream) * L.streams.size());
    up(p->d_buckets, L.buckets.data(), sizeof(uint2) * L.buckets.size());
    up(p->d_tabs, L.tabs.data(), sizeof(uint2) * L.tabs.size());
    up(p->d_syms, L.syms.data(), sizeof(uint16_t) * L.syms.size());
    up(p->d_ss, L.segs.data(), sizeof(SegStream) * L.segs.size());
    up(p->d_seg_stream, L.seg_stream.data(), sizeof(uint32_t) * L.seg_stream.size());
    if (e == cudaSuccess) e = cudaMallocHost(&p->h_errs, 4ull * n_internal);
    if (e != cudaSuccess) {
        rc = cuda_fail(e, "plan upload");
        free_plan(p);
        return rc;
    }
    *out_plan = p;
    return BS_OK;
}

int check_device(int device) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return fail(BS_E_INVALID_ARG, "invalid CUDA device " + std::to_string(device));
    }
    return BS_OK;
}

}  // namespace

extern "C" {

int bs_par_plan_create(const uint8_t *h, uint64_t len, uint64_t n_weights, const void *d_blob, void *d_out,
                       int device, bs_plan **out_plan) {
    if (!out_plan) return fail(BS_E_INVALID_ARG, "out_plan is NULL");
    *out_plan = nullptr;
    int rc = check_device(device);
    if (rc) return rc;
    DeviceGuard guard(device);
    SerialLayout L;
    // bf16_parallel.py:268-269: nothing to decode
    if (n_weights == 0 || len == 0) return make_serial_plan(L, device, 1, {-1}, 0, out_plan);
    if (!h) return fail(BS_E_INVALID_ARG, "host blob is NULL");
    if (!d_blob || !d_out || !on_device(d_blob, device) || !on_device(d_out, device))
        return fail(BS_E_INVALID_ARG, "d_blob/d_out must be device memory of device " + std::to_string(device));
    SerialBlob B{h, len, n_weights, reinterpret_cast<uint64_t>(d_blob), reinterpret_cast<uint64_t>(d_out), 0};
    rc = parse_par1(L, B);
    if (rc) return rc;
    return make_serial_plan(L, device, 1, {0}, 1, out_plan);
}

int bs_se_parse(int codec, const uint8_t *h, uint64_t len, uint64_t n_weights, uint32_t *n_jobs_out) {
    if (n_jobs_out) *n_jobs_out = 0;
    if (codec != BS_SE_SINGLE_KERNEL && codec != BS_SE_TANS && codec != BS_SE_PARALLEL)
        return fail(BS_E_INVALID_ARG, "unknown legacy codec " + std::to_string(codec));
    if (n_weights == 0 || len == 0) return BS_OK;
    if (!h) return fail(BS_E_INVALID_ARG, "host blob is NULL");
    SerialLayout L;
    SerialBlob B{h, len, n_weights, 0, 0, 0};
    const int rc = parse_serial(codec, L, B);
    if (rc == BS_OK && n_jobs_out) *n_jobs_out = static_cast<uint32_t>(L.jobs.size());
    return rc;
}

int bs_se_plan_create_many(const bs_se_blob *blobs, int n_blobs, int device, bs_plan **out_plan) {
    if (!out_plan) return fail(BS_E_INVALID_ARG, "out_plan is NULL");
    *out_plan = nullptr;
    if (n_blobs < 0 || (n_blobs > 0 && !blobs)) return fail(BS_E_INVALID_ARG, "bad blob array");
    int rc = check_device(device);
    if (rc) return rc;
    DeviceGuard guard(device);
    SerialLayout L;
    std::vector<int> u2i(n_blobs, -1);
    int n_internal = 0;
    for (int i = 0; i < n_blobs; i++) {
        const bs_se_blob &b = blobs[i];
        const std::string who = "blob " + std::to_string(i) + ": ";
        if (b.codec != BS_SE_SINGLE_KERNEL && b.codec != BS_SE_TANS && b.codec != BS_SE_PARALLEL)
            return fail(BS_E_INVALID_ARG, who + "unknown legacy codec " + std::to_string(b.codec));
        // single_kernel.py:603-613 / bf16_tans.py:121-125 / bf16_parallel.py:268-269: nothing to decode
        if (b.n_weights == 0 || b.blob_bytes == 0) continue;
        if (!b.h_blob) return fail(BS_E_INVALID_ARG, who + "host blob is NULL");
        if (!b.d_blob || !b.d_out || !on_device(b.d_blob, device) || !on_device(b.d_out, device))
            return fail(BS_E_INVALID_ARG, who + "d_blob/d_out must be device memory of device " + std::to_string(device));
        SerialBlob B{b.h_blob, b.blob_bytes, b.n_weights, reinterpret_cast<uint64_t>(b.d_blob),
                     reinterpret_cast<uint64_t>(b.d_out), static_cast<uint32_t>(n_internal)};
        rc = parse_serial(b.codec, L, B);
        if (rc) return rc;
        u2i[i] = n_internal++;
    }
    return make_serial_plan(L, device, n_blobs, u2i, n_internal, out_plan);
}

int bs_se_plan_create(int codec, const uint8_t *h, uint64_t len, uint64_t n_weights, const void *d_blob,
                      void *d_out, int device, bs_plan **out_plan) {
    const bs_se_blob b{codec, h, len, n_weights, d_blob, d_out};
    return bs_se_plan_create_many(&b, 1, device, out_plan);
}

// --------------------------------------------------------------------------
// encoder
// --------------------------------------------------------------------------
}  // extern "C"

namespace {
// values per state group, or 0 when (chunk_elems, groups) is not valid
uint32_t group_elems(uint32_t ce, uint32_t groups) {
    const uint32_t G = groups ? groups : 1u;
    if (ce == 0 || ce % G) return 0;
    const uint32_t ge = ce / G;
    return (ge >= 256 && !(ge & 255)) ? ge : 0u;
}
}  // namespace

extern "C" {

int bs_xc_encode_bound(uint64_t n, uint32_t ce, uint32_t groups, uint64_t *bytes) {
    const uint32_t ge = group_elems(ce, groups);
    if (!bytes || !ge) return fail(BS_E_INVALID_ARG, "bad encode_bound arguments");
    *bytes = n ? xc_encode_bound(n, ge) : 0;
    return BS_OK;
}

int bs_xc_encode_workspace(uint64_t n, uint32_t ce, uint32_t groups, int coder, uint64_t *bytes) {
    const uint32_t ge = group_elems(ce, groups);
    if (!bytes || !ge || coder < BS_CODER_RANS || coder > BS_CODER_RANS_PAIR)
        return fail(BS_E_INVALID_ARG, "bad encode_workspace arguments");
    *bytes = n ? xc_encode_workspace(n, ge, coder) : 0;
    return BS_OK;
}

int bs_xc_encode(const void *d_in, uint64_t n, int coder, int prec, uint32_t ce_chunk, uint32_t groups,
                 void *d_out, uint64_t out_cap, uint64_t *d_out_len, void *d_ws, uint64_t ws_bytes, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint32_t ce = group_elems(ce_chunk, groups);   // the encoder codes state groups
    const uint32_t G = groups ? groups : 1u;
    if (!ce) return fail(BS_E_INVALID_ARG, "chunk_elems / groups must be a positive multiple of 256");
    if (prec < 8 || prec > 12) return fail(BS_E_INVALID_ARG, "precision must be in [8, 12]");
    if (coder < BS_CODER_RANS || coder > BS_CODER_RANS_PAIR)
        return fail(BS_E_INVALID_ARG, "coder must be 0 (rANS), 1 (tANS) or 2 (rANS over exponent pairs)");
    if (!d_out_len) return fail(BS_E_INVALID_ARG, "d_out_len is NULL");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(BS_E_CUDA, "no current device");
    if (!on_device(d_out_len, dev)) return fail(BS_E_INVALID_ARG, "d_out_len must be device memory");
    if (n == 0) {
        cudaError_t e = cudaMemsetAsync(d_out_len, 0, 8, s);
        return e == cudaSuccess ? BS_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    if (!d_in || !d_out || !d_ws) return fail(BS_E_INVALID_ARG, "NULL pointer");
    if ((reinterpret_cast<uintptr_t>(d_in) | reinterpret_cast<uintptr_t>(d_out) |
         reinterpret_cast<uintptr_t>(d_ws) | reinterpret_cast<uintptr_t>(d_out_len)) & 15)
        return fail(BS_E_INVALID_ARG, "input, output, workspace and length must be 16-byte aligned");
    if (!on_device(d_in, dev) || !on_device(d_out, dev) || !on_device(d_ws, dev))
        return fail(BS_E_INVALID_ARG, "pointers must be device memory of the current device");
    if ((n + ce - 1) / ce > 0x7FFFFFFFull) return fail(BS_E_INVALID_ARG, "too many chunks");
    if (out_cap < xc_encode_bound(n, ce)) return fail(BS_E_INVALID_ARG, "out_cap below bs_xc_encode_bound");
    if (ws_bytes < xc_encode_workspace(n, ce, coder)) return fail(BS_E_INVALID_ARG, "workspace below bs_xc_encode_workspace");
    cudaError_t e = launch_xc_encode(static_cast<const uint16_t *>(d_in), n, coder, prec, ce, G,
                                     static_cast<uint8_t *>(d_out), out_cap, d_out_len,
                                     static_cast<uint8_t *>(d_ws), ws_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "encode launch");
    return BS_OK;
}

}  // extern "C"
