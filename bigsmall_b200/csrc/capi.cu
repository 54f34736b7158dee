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
    uint32_t *d_tables = nullptr;
    // bf16_parallel_v1
    const uint8_t *d_blob = nullptr;
    uint16_t *d_out = nullptr;
    ParJob *d_jobs = nullptr;
    int n_jobs = 0;
    ParStream *d_streams = nullptr;
    int n_streams_total = 0;
    uint32_t *d_buckets = nullptr;
    uint2 *d_se_tab = nullptr;
    uint2 *d_m_tabs = nullptr;
    uint16_t *d_se_sym = nullptr;
    uint8_t *d_mant = nullptr;
    uint32_t par_n_streams = 0;
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
    if (p->d_mem) cudaFree(p->d_mem);
    if (p->h_errs) cudaFreeHost(p->h_errs);
    delete p;
}

}  // namespace

extern "C" {

int bs_version(void) { return 100; }

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

int bs_plan_n_tensors(const bs_plan *plan) { return plan ? plan->n_tensors : 0; }

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
        const std::string who = "tensor " + std::to_string(i) + ": ";
        if (t.coder_mask & ~kXcAllCoders) return fail(BS_E_INVALID_ARG, who + "coder_mask has unknown coder bits");
        if (!t.d_blob || !t.d_out) return fail(BS_E_INVALID_ARG, who + "NULL pointer");
        if ((reinterpret_cast<uintptr_t>(t.d_blob) | reinterpret_cast<uintptr_t>(t.d_out)) & 15)
            return fail(BS_E_INVALID_ARG, who + "blob and output must be 16-byte aligned");
        if (t.chunk_elems < 256 || (t.chunk_elems & 255))
            return fail(BS_E_INVALID_ARG, who + "chunk_elems must be a positive multiple of 256");
        uint64_t nc = (t.n_elems + t.chunk_elems - 1) / t.chunk_elems;
        if (nc > 0x7FFFFFFFull) return fail(BS_E_INVALID_ARG, who + "too many chunks");
        if (t.chunk_begin >= nc) return fail(BS_E_INVALID_ARG, who + "chunk_begin beyond the last chunk");
        const uint64_t cnt = t.chunk_count ? t.chunk_count : nc - t.chunk_begin;
        if (t.chunk_begin + cnt > nc) return fail(BS_E_INVALID_ARG, who + "chunk range beyond the last chunk");
        uint64_t min_bytes = rup(kXcTabOff + 4 * (nc + 1), 16) + rup(t.n_elems, 16) + 128 * nc;
        if (t.blob_bytes < min_bytes) return fail(BS_E_TRUNCATED, who + "blob shorter than its framing");
        if (!on_device(t.d_blob, device) || !on_device(t.d_out, device))
            return fail(BS_E_INVALID_ARG, who + "pointers must be device memory of device " + std::to_string(device));
        XcTensorDev d{};
        d.blob = static_cast<const uint8_t *>(t.d_blob);
        d.blob_bytes = t.blob_bytes;
        d.out = static_cast<uint16_t *>(t.d_out);
        d.n = t.n_elems;
        d.chunk_elems = t.chunk_elems;
        d.n_chunks = static_cast<uint32_t>(nc);
        d.chunk_begin = t.chunk_begin;
        d.aux = 0;
        d.coder = 0xFFFFFFFFu;
        d.coder_mask = t.coder_mask;
        u2i[i] = static_cast<int>(ht.size());
        ht.push_back(d);
        ranges.push_back({t.chunk_begin, static_cast<uint32_t>(cnt)});
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

int bs_plan_decode(bs_plan *p, void *stream) {
    if (!p) return fail(BS_E_INVALID_ARG, "plan is NULL");
    DeviceGuard guard(p->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (p->kind == kPlanXc) {
        if (p->n_internal == 0) return BS_OK;
        e = launch_xc_prepare(p->d_tens, p->n_internal, p->d_tables, p->d_errs, s);
        if (e == cudaSuccess)
            e = launch_xc_decode(p->d_tens, p->d_items, p->n_items, p->d_tables, p->d_errs, p->coders, s);
    } else if (p->kind == kPlanPar) {
        if (p->n_internal == 0) return BS_OK;
        e = cudaMemsetAsync(p->d_errs, 0, 4, s);
        if (e == cudaSuccess)
            e = launch_par_jobs(p->d_blob, p->d_jobs, p->n_jobs, p->d_se_tab, p->d_m_tabs, p->d_se_sym,
                                p->d_mant, p->d_errs, s);
        if (e == cudaSuccess)
            e = launch_par_merge(p->d_streams, p->n_streams_total, p->d_buckets, p->d_se_sym, p->d_mant,
                                 p->d_out, p->par_n_streams, p->d_errs, s);
    } else {
        return fail(BS_E_INVALID_ARG, "unknown plan kind");
    }
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
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
        int k = p->kind == kPlanXc ? p->user_to_internal[i] : (p->n_internal ? 0 : -1);
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
        const std::string who = "tensor " + std::to_string(i) + ": ";
        if (t.coder_mask & ~kXcAllCoders) return fail(BS_E_INVALID_ARG, who + "coder_mask has unknown coder bits");
        if (!t.d_blob || !t.d_out) return fail(BS_E_INVALID_ARG, who + "NULL pointer");
        if ((reinterpret_cast<uintptr_t>(t.d_blob) | reinterpret_cast<uintptr_t>(t.d_out)) & 15)
            return fail(BS_E_INVALID_ARG, who + "blob and output must be 16-byte aligned");
        if (t.chunk_elems < 256 || (t.chunk_elems & 255))
            return fail(BS_E_INVALID_ARG, who + "chunk_elems must be a positive multiple of 256");
        const uint64_t nc = (t.n_elems + t.chunk_elems - 1) / t.chunk_elems;
        if (nc > 0x7FFFFFFFull) return fail(BS_E_INVALID_ARG, who + "too many chunks");
        if (t.chunk_begin >= nc) return fail(BS_E_INVALID_ARG, who + "chunk_begin beyond the last chunk");
        const uint64_t cnt = t.chunk_count ? t.chunk_count : nc - t.chunk_begin;
        if (t.chunk_begin + cnt > nc) return fail(BS_E_INVALID_ARG, who + "chunk range beyond the last chunk");
        const uint64_t min_bytes = rup(kXcTabOff + 4 * (nc + 1), 16) + rup(t.n_elems, 16) + 128 * nc;
        if (t.blob_bytes < min_bytes) return fail(BS_E_TRUNCATED, who + "blob shorter than its framing");
        if (!on_device(t.d_blob, device) || !on_device(t.d_out, device))
            return fail(BS_E_INVALID_ARG, who + "pointers must be device memory of the current device");
        XcTensorDev d{};
        d.blob = static_cast<const uint8_t *>(t.d_blob);
        d.blob_bytes = t.blob_bytes;
        d.out = static_cast<uint16_t *>(t.d_out);
        d.n = t.n_elems;
        d.chunk_elems = t.chunk_elems;
        d.n_chunks = static_cast<uint32_t>(nc);
        d.chunk_begin = t.chunk_begin;
        d.coder = 0xFFFFFFFFu;
        d.coder_mask = t.coder_mask;
        ht[n] = d;
        rc_count[n] = static_cast<uint32_t>(cnt);
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
int bs_par_plan_create(const uint8_t *h, uint64_t len, uint64_t n_weights, const void *d_blob, void *d_out,
                       int device, bs_plan **out_plan) {
    if (!out_plan) return fail(BS_E_INVALID_ARG, "out_plan is NULL");
    *out_plan = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return fail(BS_E_INVALID_ARG, "invalid CUDA device " + std::to_string(device));
    }
    DeviceGuard guard(device);
    auto *p = new bs_plan();
    p->kind = kPlanPar;
    p->device = device;
    p->n_tensors = 1;
    // bf16_parallel.py:268-269: nothing to decode
    if (n_weights == 0 || len == 0) {
        p->n_internal = 0;
        *out_plan = p;
        return BS_OK;
    }
    if (!h) { delete p; return fail(BS_E_INVALID_ARG, "host blob is NULL"); }
    uint64_t pos = 0;
    int rc = BS_OK;
    auto need = [&](uint64_t k) -> bool {
        if (pos + k > len) { rc = fail(BS_E_TRUNCATED, "bf16_parallel: blob truncated in header"); return false; }
        return true;
    };
    // _unpack_header (bf16_parallel.py:138-183)
    if (!need(4)) { delete p; return rc; }
    if (memcmp(h, "PAR1", 4) != 0) { delete p; return fail(BS_E_BAD_MAGIC, "bf16_parallel: bad magic"); }
    pos = 4;
    if (!need(10)) { delete p; return rc; }
    const uint64_t n = rd32(h + 4);
    const uint32_t ns = rd16(h + 8), p_se = rd16(h + 10), p_m = rd16(h + 12);
    pos = 14;
    if (p_se != 12 || p_m != 10) {
        delete p;
        return fail(BS_E_PRECISION, "bf16_parallel: precision mismatch (header SE=" + std::to_string(p_se) +
                                        " M=" + std::to_string(p_m) + " vs codec SE=12 M=10)");
    }
    if (!need(2)) { delete p; return rc; }
    const uint32_t n_se_nz = rd16(h + pos);
    pos += 2;
    if (!need(6ull * n_se_nz)) { delete p; return rc; }
    std::vector<uint32_t> se_f(512, 0);
    for (uint32_t i = 0; i < n_se_nz; i++) {
        uint32_t s = rd16(h + pos + 2 * i);
        if (s >= 512) { delete p; return fail(BS_E_CORRUPT, "bf16_parallel: SE symbol index out of range"); }
        se_f[s] = rd32(h + pos + 2ull * n_se_nz + 4 * i);
    }
    pos += 6ull * n_se_nz;
    if (!need(4)) { delete p; return rc; }
    const uint32_t n_exps = rd32(h + pos);
    pos += 4;
    if (!need(2ull * n_exps)) { delete p; return rc; }
    std::vector<int> exp_tab(256, -1);
    std::vector<std::vector<uint32_t>> mfreq;
    const uint64_t exps_pos = pos;
    pos += 2ull * n_exps;
    for (uint32_t q = 0; q < n_exps; q++) {
        uint32_t ev = rd16(h + exps_pos + 2 * q);
        if (!need(1)) { delete p; return rc; }
        uint32_t nzc = h[pos];
        pos += 1;
        if (!need(5ull * nzc)) { delete p; return rc; }
        if (ev >= 256) { delete p; return fail(BS_E_CORRUPT, "bf16_parallel: exponent out of range"); }
        std::vector<uint32_t> mf(128, 0);
        for (uint32_t i = 0; i < nzc; i++) {
            uint32_t m = h[pos + i];
            if (m >= 128) { delete p; return fail(BS_E_CORRUPT, "bf16_parallel: mantissa index out of range"); }
            mf[m] = rd32(h + pos + nzc + 4 * i);
        }
        pos += 5ull * nzc;
        if (exp_tab[ev] < 0) {
            exp_tab[ev] = static_cast<int>(mfreq.size());
            mfreq.push_back(mf);
        } else {
            mfreq[exp_tab[ev]] = mf;   // later entries overwrite (dict semantics)
        }
    }
    if (n != n_weights) {
        delete p;
        return fail(BS_E_COUNT_MISMATCH, "bf16_parallel: weight count mismatch (" + std::to_string(n) + " vs " +
                                             std::to_string(n_weights) + ")");
    }
    if (ns == 0) { delete p; return fail(BS_E_CORRUPT, "bf16_parallel: zero streams"); }
    if (!d_blob || !d_out || !on_device(d_blob, device) || !on_device(d_out, device)) {
        delete p;
        return fail(BS_E_INVALID_ARG, "d_blob/d_out must be device memory of device " + std::to_string(device));
    }
    const uint64_t header_end = pos;
    const uint64_t n_off = static_cast<uint64_t>(ns) + 1;
    if (header_end + 4 * n_off > len) { delete p; return fail(BS_E_TRUNCATED, "bf16_parallel: offset table truncated"); }
    const uint8_t *offt = h + header_end;
    const uint64_t payload_start = header_end + 4 * n_off;

    // decode tables: slot -> {sym | freq[sym] << 16, cum[sym]}; unassigned slots
    // map to symbol 0 like rans.build_slot_to_symbol's zero-initialised table
    auto build_tab = [](const std::vector<uint32_t> &f, uint32_t M, std::vector<uint2> &tab) {
        std::vector<uint32_t> cum(f.size());
        uint64_t c = 0;
        for (size_t s = 0; s < f.size(); s++) { cum[s] = static_cast<uint32_t>(c); c += f[s]; }
        tab.assign(M, make_uint2(0u | (std::min<uint32_t>(f[0], 0xFFFF) << 16), cum[0]));
        for (size_t s = 0; s < f.size(); s++)
            for (uint64_t j = 0; j < f[s] && cum[s] + j < M; j++)
                tab[cum[s] + j] = make_uint2(static_cast<uint32_t>(s) | (std::min<uint32_t>(f[s], 0xFFFF) << 16), cum[s]);
    };
    std::vector<uint2> se_tab, m_tabs;
    build_tab(se_f, 4096, se_tab);
    for (auto &mf : mfreq) {
        std::vector<uint2> t;
        build_tab(mf, 1024, t);
        m_tabs.insert(m_tabs.end(), t.begin(), t.end());
    }
    for (uint32_t v : se_f)
        if (v > 0xFFFF) { delete p; return fail(BS_E_CORRUPT, "bf16_parallel: SE frequency out of range"); }

    std::vector<ParJob> jobs;
    std::vector<ParStream> streams;
    std::vector<uint2> buckets;
    uint64_t se_cur = 0;
    for (uint32_t k = 0; k < ns; k++) {
        const uint64_t nin = k < n ? (n - 1 - k) / ns + 1 : 0;
        if (nin == 0) continue;
        uint64_t a = payload_start + rd32(offt + 4ull * k), b = payload_start + rd32(offt + 4ull * (k + 1));
        a = std::min(a, len);
        b = std::min(b, len);
        if (b < a) b = a;
        uint64_t q = a;
        const std::string who = "bf16_parallel: stream " + std::to_string(k) + ": ";
        if (q + 4 > b) { delete p; return fail(BS_E_TRUNCATED, who + "truncated"); }
        const uint32_t se_len = rd32(h + q);
        q += 4;
        const uint64_t se_got = std::min<uint64_t>(se_len, b - q);
        ParJob sej{q, static_cast<uint32_t>(se_got), static_cast<uint32_t>(nin), se_cur, 0, 1};
        jobs.push_back(sej);
        q += se_got;
        if (q + 4 > b) { delete p; return fail(BS_E_TRUNCATED, who + "truncated"); }
        const uint32_t nze = rd32(h + q);
        q += 4;
        if (q + 2ull * nze > b) { delete p; return fail(BS_E_TRUNCATED, who + "truncated"); }
        const uint64_t sx = q;
        q += 2ull * nze;
        ParStream S{};
        S.se_off = se_cur;
        S.mant_off = se_cur;
        S.n_in = static_cast<uint32_t>(nin);
        S.k = k;
        S.bucket_first = static_cast<uint32_t>(buckets.size());
        S.n_buckets = nze;
        std::vector<uint64_t> cnt(256, 0);
        std::vector<uint8_t> seen(256, 0);
        std::vector<std::pair<uint32_t, ParJob>> bj;
        uint64_t total = 0;
        for (uint32_t qq = 0; qq < nze; qq++) {
            const uint32_t ev = rd16(h + sx + 2ull * qq);
            if (q + 8 > b) { delete p; return fail(BS_E_TRUNCATED, who + "truncated"); }
            const uint32_t count = rd32(h + q), blen = rd32(h + q + 4);
            q += 8;
            const uint64_t got = std::min<uint64_t>(blen, b - q);
            if (ev >= 256 || exp_tab[ev] < 0) { delete p; return fail(BS_E_CORRUPT, who + "bucket exponent has no table"); }
            if (seen[ev]) { delete p; return fail(BS_E_CORRUPT, who + "duplicate bucket exponent"); }
            seen[ev] = 1;
            cnt[ev] = count;
            total += count;
            ParJob mj{q, static_cast<uint32_t>(got), count, 0, static_cast<uint32_t>(exp_tab[ev]) + 1, 0};
            bj.push_back({ev, mj});
            buckets.push_back(make_uint2(ev, count));
            q += got;
        }
        if (total != nin) { delete p; return fail(BS_E_CORRUPT, who + "bucket counts do not sum to the stream size"); }
        std::vector<uint64_t> bstart(257, 0);
        for (int e = 0; e < 256; e++) bstart[e + 1] = bstart[e] + cnt[e];
        for (auto &x : bj) {
            x.second.out_off = S.mant_off + bstart[x.first];
            jobs.push_back(x.second);
        }
        streams.push_back(S);
        se_cur += nin;
    }
    std::stable_sort(jobs.begin(), jobs.end(), [](const ParJob &x, const ParJob &y) { return x.n_syms > y.n_syms; });
    if (jobs.size() > 0x7FFFFFFFull || streams.size() > 0x7FFFFFFFull) {
        delete p;
        return fail(BS_E_INVALID_ARG, "too many streams");
    }
    Carve cv;
    const uint64_t o_j = cv.take(sizeof(ParJob) * jobs.size());
    const uint64_t o_s = cv.take(sizeof(ParStream) * streams.size());
    const uint64_t o_b = cv.take(sizeof(uint2) * std::max<size_t>(1, buckets.size()));
    const uint64_t o_st = cv.take(sizeof(uint2) * se_tab.size());
    const uint64_t o_mt = cv.take(sizeof(uint2) * std::max<size_t>(1, m_tabs.size()));
    const uint64_t o_ss = cv.take(2 * n);
    const uint64_t o_m = cv.take(n);
    const uint64_t o_e = cv.take(4);
    rc = alloc_plan_mem(p, cv.off);
    if (rc) { free_plan(p); return rc; }
    auto *base = static_cast<uint8_t *>(p->d_mem);
    p->d_blob = static_cast<const uint8_t *>(d_blob);
    p->d_out = static_cast<uint16_t *>(d_out);
    p->d_jobs = reinterpret_cast<ParJob *>(base + o_j);
    p->n_jobs = static_cast<int>(jobs.size());
    p->d_streams = reinterpret_cast<ParStream *>(base + o_s);
    p->n_streams_total = static_cast<int>(streams.size());
    p->d_buckets = reinterpret_cast<uint32_t *>(base + o_b);
    p->d_se_tab = reinterpret_cast<uint2 *>(base + o_st);
    p->d_m_tabs = reinterpret_cast<uint2 *>(base + o_mt);
    p->d_se_sym = reinterpret_cast<uint16_t *>(base + o_ss);
    p->d_mant = base + o_m;
    p->d_errs = reinterpret_cast<uint32_t *>(base + o_e);
    p->par_n_streams = ns;
    p->n_internal = 1;
    cudaError_t e = cudaSuccess;
    auto up = [&](void *dst, const void *src, size_t bytes) {
        if (e == cudaSuccess && bytes) e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    };
    up(p->d_jobs, jobs.data(), sizeof(ParJob) * jobs.size());
    up(p->d_streams, streams.data(), sizeof(ParStream) * streams.size());
    up(p->d_buckets, buckets.data(), sizeof(uint2) * buckets.size());
    up(p->d_se_tab, se_tab.data(), sizeof(uint2) * se_tab.size());
    up(p->d_m_tabs, m_tabs.data(), sizeof(uint2) * m_tabs.size());
    if (e == cudaSuccess) e = cudaMallocHost(&p->h_errs, 4);
    if (e != cudaSuccess) {
        rc = cuda_fail(e, "plan upload");
        free_plan(p);
        return rc;
    }
    *out_plan = p;
    return BS_OK;
}

// --------------------------------------------------------------------------
// encoder
// --------------------------------------------------------------------------
int bs_xc_encode_bound(uint64_t n, uint32_t ce, uint64_t *bytes) {
    if (!bytes || ce < 256 || (ce & 255)) return fail(BS_E_INVALID_ARG, "bad encode_bound arguments");
    *bytes = n ? xc_encode_bound(n, ce) : 0;
    return BS_OK;
}

int bs_xc_encode_workspace(uint64_t n, uint32_t ce, int coder, uint64_t *bytes) {
    if (!bytes || ce < 256 || (ce & 255) || coder < BS_CODER_RANS || coder > BS_CODER_RANS_PAIR)
        return fail(BS_E_INVALID_ARG, "bad encode_workspace arguments");
    *bytes = n ? xc_encode_workspace(n, ce, coder) : 0;
    return BS_OK;
}

int bs_xc_encode(const void *d_in, uint64_t n, int coder, int prec, uint32_t ce, void *d_out, uint64_t out_cap,
                 uint64_t *d_out_len, void *d_ws, uint64_t ws_bytes, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (ce < 256 || (ce & 255)) return fail(BS_E_INVALID_ARG, "chunk_elems must be a positive multiple of 256");
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
    cudaError_t e = launch_xc_encode(static_cast<const uint16_t *>(d_in), n, coder, prec, ce,
                                     static_cast<uint8_t *>(d_out), out_cap, d_out_len,
                                     static_cast<uint8_t *>(d_ws), ws_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "encode launch");
    return BS_OK;
}

int bs_stream_probe(const void *d_in, void *d_out, uint64_t units, int rd, int wr, int grid, void *stream) {
    if (!((rd == 1 && wr == 1) || (rd == 2 && wr == 3) || (rd == 0 && wr == 1)))
        return fail(BS_E_INVALID_ARG, "bs_stream_probe: (rd, wr) must be (1,1), (2,3) or (0,1)");
    if (grid <= 0 || units == 0 || (rd && !d_in) || !d_out) return fail(BS_E_INVALID_ARG, "bs_stream_probe: bad arguments");
    if ((reinterpret_cast<uintptr_t>(d_in) | reinterpret_cast<uintptr_t>(d_out)) & 15)
        return fail(BS_E_INVALID_ARG, "bs_stream_probe: buffers must be 16-byte aligned");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return fail(BS_E_CUDA, "no current CUDA device");
    }
    if ((rd && !on_device(d_in, device)) || !on_device(d_out, device))
        return fail(BS_E_INVALID_ARG, "bs_stream_probe: buffers must be device memory of the current device");
    cudaError_t e = launch_stream_mix(d_in, d_out, units, rd, wr, grid, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "bs_stream_probe");
    return BS_OK;
}

}  // extern "C"
