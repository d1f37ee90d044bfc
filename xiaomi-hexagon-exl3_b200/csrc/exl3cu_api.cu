// C ABI of libexl3cu (include/exl3cu.h): validation, persistent weight
// handles, workspace management and launches.  Mirrors the argument checks of
// the reference's device operator op_exl3_matmul (src/exl3-htp.c:160-190) and
// codec (src/exl3_codec.cpp:12-19, 117-135), returning status codes instead of
// asserting or throwing.
#include "exl3cu.h"
#include "exl3cu_internal.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <algorithm>
#include <climits>
#include <tuple>
#include <vector>
#include <cstdlib>

using namespace exl3cu;

struct exl3cu_weight {
    int device;
    bool model_owned;    // freed with its model handle, not by exl3cu_weight_free
    size_t k;
    size_t n_total;
    size_t first_block;
    size_t nblocks;
    unsigned bits;
    unsigned codebook;
    int sms;
    uint32_t * lsc;
    __half * su;
    __half * sv;
    void * ws;           // unused: kept null (the cluster kernel needs no workspace)
    size_t ws_bytes;     // workspace size of the global split-K variant (exl3cu_mul_mat_ws)
    GemvPlan plan;       // for rows = 8 (cps/splits do not depend on rows)
    void * stage_x;      // host-form staging
    size_t stage_x_bytes;
    float * stage_y;
    size_t stage_y_bytes;
    std::vector<void *> retired;  // outgrown staging, kept until the handle is freed (graphs may hold it)
    void * pin_x;        // synchronous small host-form calls: mapped pinned host staging the kernels
    float * pin_y;       // read and write directly (no copy engine round trips)
    size_t pin_x_bytes, pin_y_bytes;
    void * pin_x_dev;    // their device addresses
    float * pin_y_dev;
};

namespace {

thread_local std::string g_last_error;

int fail(int status, const char * fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char * what) {
    (void)cudaGetLastError();  // clear a non-sticky error so the context stays usable
    return fail(e == cudaErrorMemoryAllocation ? EXL3CU_OUT_OF_MEMORY : EXL3CU_CUDA_ERROR, "%s: %s", what,
                cudaGetErrorString(e));
}

#define CU_TRY(expr, what)                                     \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return cuda_fail(_e, (what));   \
    } while (0)

bool valid_codec(unsigned bits, unsigned cb) { return bits >= 1 && bits <= 8 && cb <= 2; }

bool valid_shape(size_t k, size_t n, size_t multiple) {
    return k && n && k % multiple == 0 && n % multiple == 0 && k <= SIZE_MAX / n;
}

// A device pointer of `device` (or managed memory); rejects host pointers,
// which a kernel could not dereference.
int check_device_ptr(const void * p, int device, const char * name) {
    if (!p) return fail(EXL3CU_INVALID_ARGUMENT, "%s is NULL", name);
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return fail(EXL3CU_INVALID_ARGUMENT, "%s is not a CUDA pointer", name);
    }
    if (attr.type == cudaMemoryTypeManaged) return EXL3CU_OK;
    if (attr.type != cudaMemoryTypeDevice)
        return fail(EXL3CU_INVALID_ARGUMENT, "%s must be device memory (got host/unregistered memory)", name);
    if (device >= 0 && attr.device != device)
        return fail(EXL3CU_INVALID_ARGUMENT, "%s lives on device %d, expected device %d", name, attr.device, device);
    return EXL3CU_OK;
}

int current_device(int * dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    return EXL3CU_OK;
}

// Makes `device` current for the scope and restores the caller's device after.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
        if (prev != device && cudaSetDevice(device) != cudaSuccess) ok = false;
    }
    ~DeviceGuard() {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int device_sms(int device) {
    static std::mutex mu;
    static int cache[64] = {0};
    std::lock_guard<std::mutex> g(mu);
    if (device < 0 || device >= 64) return 148;
    if (!cache[device]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
        cache[device] = v;
    }
    return cache[device];
}

void release(exl3cu_weight * w) {
    if (!w) return;
    DeviceGuard g(w->device);
    cudaFree(w->lsc);
    cudaFree(w->su);
    cudaFree(w->sv);
    cudaFree(w->ws);
    cudaFree(w->stage_x);
    cudaFree(w->stage_y);
    for (void * p : w->retired) cudaFree(p);
    if (w->pin_x) cudaFreeHost(w->pin_x);
    if (w->pin_y) cudaFreeHost(w->pin_y);
    delete w;
}

// Common tail of the two loaders: allocate, plan, zero the workspace.
int make_weight(size_t k, size_t n, unsigned bits, unsigned cb, size_t first_block, size_t block_count, int device,
                exl3cu_weight ** out, exl3cu_weight ** made) {
    if (!out) return fail(EXL3CU_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (!valid_codec(bits, cb)) return fail(EXL3CU_INVALID_ARGUMENT, "bits must be 1..8 and codebook 0..2");
    if (!valid_shape(k, n, 128)) return fail(EXL3CU_INVALID_ARGUMENT, "k and n must be nonzero multiples of 128");
    if (k > 65536 || n > 1048576)
        return fail(EXL3CU_NO_SUPPORT, "k <= 65536 and n <= 1048576 (the reference operator's limits)");
    const size_t nb_all = n / 128;
    if (block_count == 0) block_count = nb_all - (first_block < nb_all ? first_block : nb_all);
    if (first_block >= nb_all || block_count == 0 || block_count > nb_all - first_block)
        return fail(EXL3CU_INVALID_ARGUMENT, "column block range [%zu, +%zu) outside %zu blocks", first_block,
                    block_count, nb_all);
    int ndev = 0;
    CU_TRY(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
    if (device < 0 || device >= ndev) return fail(EXL3CU_INVALID_ARGUMENT, "device %d not present", device);
    auto * w = new (std::nothrow) exl3cu_weight();
    if (!w) return fail(EXL3CU_OUT_OF_MEMORY, "host allocation");
    w->device = device;
    w->k = k;
    w->n_total = n;
    w->first_block = first_block;
    w->nblocks = block_count;
    w->bits = bits;
    w->codebook = cb;
    w->sms = device_sms(device);
    w->plan = plan_gemv(w->sms, k, block_count, 8);
    w->ws_bytes = gemv_workspace_bytes(block_count, w->plan.splits);
    const size_t lsc_bytes = block_count * (k / 16) * 256u * bits;
    cudaError_t e = cudaMalloc(&w->lsc, lsc_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->su, k * sizeof(__half));
    if (e == cudaSuccess) e = cudaMalloc(&w->sv, block_count * 128 * sizeof(__half));
    if (e != cudaSuccess) {
        release(w);
        return cuda_fail(e, "allocating device weights");
    }
    *made = w;
    return EXL3CU_OK;
}

int validate_mm(const exl3cu_weight * w, const void * x, int x_dtype, size_t rows, size_t x_stride, const float * y,
                size_t y_stride) {
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    if (x_dtype != EXL3CU_F32 && x_dtype != EXL3CU_F16)
        return fail(EXL3CU_INVALID_ARGUMENT, "x dtype must be F32 (0) or F16 (1)");
    if (!rows) return fail(EXL3CU_INVALID_ARGUMENT, "rows must be >= 1");
    const size_t n_local = w->nblocks * 128;
    if (x_stride < w->k || y_stride < n_local) return fail(EXL3CU_INVALID_ARGUMENT, "row stride shorter than a row");
    if (x_stride % 4 || y_stride % 4) return fail(EXL3CU_INVALID_ARGUMENT, "row strides must be multiples of 4 elements");
    const size_t xa = x_dtype == EXL3CU_F32 ? 16 : 8;
    if (reinterpret_cast<uintptr_t>(x) % xa) return fail(EXL3CU_INVALID_ARGUMENT, "x must be %zu-byte aligned", xa);
    if (reinterpret_cast<uintptr_t>(y) % 16) return fail(EXL3CU_INVALID_ARGUMENT, "y must be 16-byte aligned");
    return EXL3CU_OK;
}

int run_mm(const exl3cu_weight * w, const void * x, int x_dtype, size_t rows, size_t x_stride, float * y,
           size_t y_stride, void * ws, cudaStream_t st) {
    GemvArgs a{};
    a.lsc = w->lsc;
    a.su = w->su;
    a.sv = w->sv;
    a.x_f16 = x_dtype == EXL3CU_F16;
    a.x_stride = (long long)x_stride;
    a.y_stride = (long long)y_stride;
    a.nblocks = int(w->nblocks);
    a.nchunks = int(w->k / 16);
    a.cps = w->plan.cps;
    a.splits = w->plan.splits;
    if (a.splits > 1) {
        a.ws_partial = static_cast<float *>(ws);
        a.ws_count = reinterpret_cast<unsigned *>(static_cast<char *>(ws) + w->nblocks * size_t(a.splits) * 8 * 128 *
                                                                               sizeof(float));
    }
    const size_t es = x_dtype == EXL3CU_F32 ? 4 : 2;
    for (size_t r0 = 0; r0 < rows; r0 += 8) {
        const int rb = int(rows - r0 < 8 ? rows - r0 : 8);
        GemvPlan p = plan_gemv(w->sms, w->k, w->nblocks, rb);
        p.cps = w->plan.cps;
        p.splits = w->plan.splits;
        a.rows = rb;
        a.x = static_cast<const char *>(x) + r0 * x_stride * es;
        a.y = y + r0 * y_stride;
        cudaError_t e = launch_gemv(a, p, w->bits, w->codebook, st);
        if (e != cudaSuccess) return cuda_fail(e, "launching the EXL3 GEMV");
    }
    return EXL3CU_OK;
}


// One operand set of a grouped launch.
struct MmItem {
    const exl3cu_weight * w;
    const void * x;
    int x_dtype;
    size_t rows;
    size_t x_stride;
    float * y;
    size_t y_stride;
    int x_mode = kXPlain;       // kXGlu / kXRmsNorm: fused input forms (mul1 GEMV only)
    const float * nw = nullptr;  // kXRmsNorm weights [k]
    float eps = 0.f;
    int y_accum = 0;
    const float * x_ss = nullptr;  // kXRmsNorm: the rows' per-128-block sums of squares [rows][k/128]
    float * y_ss = nullptr;        // per-128-block sums of squares of the final y [rows][n_local/128]
};

bool pdl_enabled() {
    static const bool on = [] {
        const char * env = std::getenv("EXL3CU_PDL");
        return !(env && env[0] == '0');
    }();
    return on;
}

// Row count from which an operand goes to the tensor-core GEMM instead of the
// row-by-row GEMV kernels, and the plan overrides of exl3cu_gemm_config.
std::atomic<size_t> g_gemm_min_rows{5};
std::atomic<int> g_gemm_tokens{0};
std::atomic<int> g_gemm_splits{0};

size_t gemm_min_rows() { return g_gemm_min_rows.load(std::memory_order_relaxed); }

// Tiled-activation scratch of the GEMM, one buffer per (device, stream) so
// that operators on different streams never share it; work on one stream is
// ordered, so consecutive calls reuse it.  When a call needs more it gets a
// larger buffer and the old one is retired, not freed: a CUDA graph captured
// earlier on the stream keeps its pointer, and every such pointer stays valid
// for the life of the process (growth is geometric, so retired buffers add at
// most the size of the live one).  Growth allocates, which is refused while the
// stream is being captured: run one call of the largest row count first.
struct GemmScratch {
    int device;
    cudaStream_t stream;
    void * ptr;
    size_t bytes;
    std::vector<void *> retired;
};
std::mutex g_gemm_scratch_mu;
std::vector<GemmScratch> g_gemm_scratch;

int gemm_scratch(int device, cudaStream_t st, size_t bytes, void ** out) {
    std::lock_guard<std::mutex> lock(g_gemm_scratch_mu);
    GemmScratch * s = nullptr;
    for (auto & e : g_gemm_scratch)
        if (e.device == device && e.stream == st) s = &e;
    if (!s) {
        g_gemm_scratch.push_back(GemmScratch{device, st, nullptr, 0, {}});
        s = &g_gemm_scratch.back();
    }
    if (s->bytes < bytes) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        CU_TRY(cudaStreamIsCapturing(st, &cs), "querying stream capture");
        if (cs != cudaStreamCaptureStatusNone)
            return fail(EXL3CU_NO_SUPPORT,
                        "the GEMM scratch must grow to %zu bytes during stream capture: run one call with this many "
                        "rows on the stream before capturing", bytes);
        const size_t want = bytes > 2 * s->bytes ? bytes : 2 * s->bytes;
        void * p = nullptr;
        CU_TRY(cudaMalloc(&p, want), "allocating the GEMM scratch");
        if (s->ptr) s->retired.push_back(s->ptr);
        s->ptr = p;
        s->bytes = want;
    }
    *out = s->ptr;
    return EXL3CU_OK;
}

// Limits of the ragged entries (sequences per batch, packed rows per batch).
constexpr size_t kMaxRaggedSeqs = 65536;
constexpr int32_t kMaxRaggedRows = 1 << 20;

// Ids per get_rows call (the launch grid's y extent is 65535).
constexpr size_t kMaxGetRows = 65535;

// Grow one of a handle's host-form staging buffers to at least `want` bytes.
// The outgrown buffer is retired, not freed: work still in flight, or a
// captured graph, may reference it until the handle is freed.
int grow_stage(exl3cu_weight * w, void ** buf, size_t * bytes, size_t want) {
    if (*bytes >= want) return EXL3CU_OK;
    void * p = nullptr;
    const cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) return cuda_fail(e, "allocating host-form staging");
    if (*buf) w->retired.push_back(*buf);
    *buf = p;
    *bytes = want;
    return EXL3CU_OK;
}

// Mapped pinned host staging (zero-copy) for synchronous host-form calls; grown on demand (a grow
// synchronises the device, which a synchronous call does anyway).
int grow_pinned(void ** buf, size_t * bytes, size_t want) {
    if (*bytes >= want) return EXL3CU_OK;
    if (*buf) {
        cudaError_t e = cudaFreeHost(*buf);
        *buf = nullptr;
        *bytes = 0;
        if (e != cudaSuccess) return cuda_fail(e, "freeing outgrown pinned staging");
    }
    void * p = nullptr;
    const cudaError_t e = cudaHostAlloc(&p, want, cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return cuda_fail(e, "allocating pinned host staging");
    *buf = p;
    *bytes = want;
    return EXL3CU_OK;
}

// Rows at most which a synchronous host-form call runs zero-copy (decode-sized operands).
constexpr size_t kZeroCopyRows = 8;

// Rows per GEMM launch pair: bounds the scratch (2 KB per row per 1024 of k)
// and keeps every index of the launch in 32 bits.
constexpr size_t kGemmRowsPerLaunch = 2048;

// The tensor-core GEMM over `it`'s rows in launch pairs of at most
// kGemmRowsPerLaunch rows.  With m_dev set, it.rows is the capacity and the
// live row count is read on the device (ragged batches).
int run_gemm(const MmItem & it, cudaStream_t st, const int32_t * m_dev = nullptr, const PeerOut * peer = nullptr) {
    const exl3cu_weight * w = it.w;
    DeviceGuard guard(w->device);
    const size_t es = it.x_dtype == EXL3CU_F32 ? 4 : 2;
    for (size_t r0 = 0; r0 < it.rows; r0 += kGemmRowsPerLaunch) {
        const int rows = int(it.rows - r0 < kGemmRowsPerLaunch ? it.rows - r0 : kGemmRowsPerLaunch);
        const void * x = static_cast<const char *>(it.x) + r0 * it.x_stride * es;
        float * y = it.y + r0 * it.y_stride;
        const GemmPlan p = plan_gemm(w->device, w->sms, w->k, w->nblocks, w->bits, w->codebook, rows,
                                     g_gemm_tokens.load(std::memory_order_relaxed),
                                     g_gemm_splits.load(std::memory_order_relaxed));
        void * xt = nullptr;
        int rc = gemm_scratch(w->device, st, p.xt_bytes, &xt);
        if (rc) return rc;
        const cudaError_t e = launch_gemm(p, w->lsc, w->su, w->sv, w->k, w->nblocks, w->bits, w->codebook, w->device,
                                          x, it.x_dtype == EXL3CU_F16, (long long)it.x_stride, rows, m_dev, int(r0),
                                          y, (long long)it.y_stride, static_cast<__half *>(xt), pdl_enabled(), st, peer);
        if (e != cudaSuccess) return cuda_fail(e, "launching the EXL3 tensor-core GEMM");
    }
    return EXL3CU_OK;
}

// Grouped GEMV on the cluster kernels: rows beyond a problem's share become
// extra problems on the same weight; problems sharing (bits, codebook) go out
// together, at most kMaxBatch per launch, in the order given.  Operands with
// gemm_min_rows() rows or more run on the tensor-core GEMM instead, one
// launch pair each.
int run_cluster(const MmItem * items, size_t count, cudaStream_t st, const PeerOut * peer = nullptr) {
    std::vector<MmItem> gemv_items;
    gemv_items.reserve(count);
    for (size_t i = 0; i < count; ++i) {
        if (items[i].rows >= gemm_min_rows()) {
            if (items[i].x_mode != kXPlain || items[i].y_accum || items[i].y_ss)
                return fail(EXL3CU_NO_SUPPORT, "fused input forms and accumulation run on the GEMV (rows < %zu)",
                            gemm_min_rows());
            int rc = run_gemm(items[i], st);
            if (rc) return rc;
        } else {
            gemv_items.push_back(items[i]);
        }
    }
    items = gemv_items.data();
    count = gemv_items.size();
    struct Sub {
        const exl3cu_weight * w;
        const void * x;
        float * y;
        size_t x_stride, y_stride;
        int rows, x_f16;
        int x_mode, y_accum;
        const float * nw;
        float eps;
        const float * x_ss;
        float * y_ss;
    };
    std::vector<Sub> subs;
    for (size_t i = 0; i < count; ++i) {
        const MmItem & it = items[i];
        const size_t es = it.x_dtype == EXL3CU_F32 ? 4 : 2;
        // the mul1 kernel takes 4 rows per problem (two activation digits each), the other 8
        const size_t per = mul1_supported(it.w->bits, 1) && it.w->codebook == EXL3CU_CB_MUL1 ? 4 : 8;
        for (size_t r0 = 0; r0 < it.rows; r0 += per) {
            Sub s;
            s.w = it.w;
            s.x = static_cast<const char *>(it.x) + r0 * it.x_stride * es;
            s.y = it.y + r0 * it.y_stride;
            s.x_stride = it.x_stride;
            s.y_stride = it.y_stride;
            s.rows = int(it.rows - r0 < per ? it.rows - r0 : per);
            s.x_f16 = it.x_dtype == EXL3CU_F16;
            s.x_mode = it.x_mode;
            s.y_accum = it.y_accum;
            s.nw = it.nw;
            s.eps = it.eps;
            s.x_ss = it.x_ss ? it.x_ss + r0 * (it.w->k / 128) : nullptr;
            s.y_ss = it.y_ss ? it.y_ss + r0 * it.w->nblocks : nullptr;
            subs.push_back(s);
        }
    }
    std::vector<bool> done(subs.size(), false);
    for (size_t i = 0; i < subs.size(); ++i) {
        if (done[i]) continue;
        const unsigned bits = subs[i].w->bits, cb = subs[i].w->codebook;
        const int device = subs[i].w->device;
        std::vector<size_t> group;
        for (size_t j = i; j < subs.size() && group.size() < size_t(kMaxBatch); ++j)
            if (!done[j] && subs[j].w->bits == bits && subs[j].w->codebook == cb && subs[j].w->device == device) {
                group.push_back(j);
                done[j] = true;
            }
        GemvBatch b{};
        int units = 0, min_nchunks = 1 << 30, max_rows = 1;
        for (size_t gi = 0; gi < group.size(); ++gi) {
            const Sub & s = subs[group[gi]];
            GemvProblem & P = b.prob[gi];
            P.lsc = s.w->lsc;
            P.su = s.w->su;
            P.sv = s.w->sv;
            P.x = s.x;
            P.y = s.y;
            P.x_stride = (long long)s.x_stride;
            P.y_stride = (long long)s.y_stride;
            P.nchunks = int(s.w->k / 16);
            P.rows = s.rows;
            P.x_f16 = s.x_f16;
            P.x_mode = s.x_mode;
            P.nw = s.nw;
            P.eps = s.eps;
            P.y_accum = s.y_accum;
            P.x_ss = s.x_ss;
            P.y_ss = s.y_ss;
            P.y_ss_stride = int(s.w->nblocks);
            P.unit_base = units;
            units += int(s.w->nblocks);
            min_nchunks = P.nchunks < min_nchunks ? P.nchunks : min_nchunks;
            max_rows = s.rows > max_rows ? s.rows : max_rows;
        }
        b.count = int(group.size());
        if (peer) {  // one 1..4-row mul1 problem (checked by the caller)
            b.peer_on = 1;
            b.peer = *peer;
        }
        if (cb == EXL3CU_CB_MUL1 && mul1_supported(bits, max_rows)) {
            DeviceGuard guard(device);
            cudaError_t e = launch_gemv_mul1(b, units, subs[i].w->sms, device, bits, pdl_enabled(), st);
            if (e != cudaSuccess) return cuda_fail(e, "launching the EXL3 mul1 GEMV");
            continue;
        }
        for (size_t gi = 0; gi < group.size(); ++gi)
            if (subs[group[gi]].x_mode != kXPlain || subs[group[gi]].y_accum || subs[group[gi]].y_ss)
                return fail(EXL3CU_NO_SUPPORT, "fused input forms and accumulation need mul1 weights of 2..8 bits");
        b.splits = choose_cluster_splits(subs[i].w->sms, units, min_nchunks);
        int max_cps = 1;
        for (int gi = 0; gi < b.count; ++gi) {
            b.prob[gi].cps = (b.prob[gi].nchunks + b.splits - 1) / b.splits;
            max_cps = b.prob[gi].cps > max_cps ? b.prob[gi].cps : max_cps;
        }
        const size_t smem = cluster_smem_bytes(max_cps, max_rows);
        if (smem > 200 * 1024) return fail(EXL3CU_NO_SUPPORT, "K range per cluster rank too long (%d chunks)", max_cps);
        DeviceGuard guard(device);
        cudaError_t e = launch_gemv_cluster(b, units, smem, bits, cb, pdl_enabled(), st);
        if (e != cudaSuccess) return cuda_fail(e, "launching the EXL3 cluster GEMV");
    }
    return EXL3CU_OK;
}

}  // namespace

extern "C" {

int exl3cu_abi_version(void) { return EXL3CU_ABI_VERSION; }

const char * exl3cu_status_string(int status) {
    switch (status) {
        case EXL3CU_OK: return "ok";
        case EXL3CU_INVALID_ARGUMENT: return "invalid argument";
        case EXL3CU_NO_SUPPORT: return "not supported";
        case EXL3CU_OUT_OF_MEMORY: return "out of device memory";
        case EXL3CU_CUDA_ERROR: return "CUDA error";
        default: return "unknown status";
    }
}

const char * exl3cu_last_error(void) { return g_last_error.c_str(); }

int exl3cu_decode_codebook(const uint16_t * d_states, size_t count, unsigned codebook, uint16_t * d_out,
                           void * stream) {
    if (codebook > 2) return fail(EXL3CU_INVALID_ARGUMENT, "Unknown EXL3 codebook");
    if (!count) return EXL3CU_OK;
    int dev, rc;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = check_device_ptr(d_states, dev, "states"))) return rc;
    if ((rc = check_device_ptr(d_out, dev, "out"))) return rc;
    CU_TRY(launch_codebook(d_states, count, codebook, d_out, static_cast<cudaStream_t>(stream)), "codebook kernel");
    return EXL3CU_OK;
}

int exl3cu_decode_inner(const uint16_t * d_packed, size_t k, size_t n, size_t first_column, size_t column_count,
                        unsigned bits, unsigned codebook, uint16_t * d_out, void * stream) {
    if (!valid_codec(bits, codebook)) return fail(EXL3CU_INVALID_ARGUMENT, "EXL3 integer bitrate must be in [1,8]");
    if (!valid_shape(k, n, 16)) return fail(EXL3CU_INVALID_ARGUMENT, "Invalid EXL3 matrix dimensions");
    if (!column_count || first_column % 16 || column_count % 16 || first_column > n ||
        column_count > n - first_column)
        return fail(EXL3CU_INVALID_ARGUMENT, "Invalid EXL3 column slice");
    int dev, rc;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = check_device_ptr(d_packed, dev, "packed"))) return rc;
    if ((rc = check_device_ptr(d_out, dev, "out"))) return rc;
    if (reinterpret_cast<uintptr_t>(d_out) % 16) return fail(EXL3CU_INVALID_ARGUMENT, "out must be 16-byte aligned");
    CU_TRY(launch_decode_inner(d_packed, k, n, first_column, column_count, bits, codebook, d_out,
                               static_cast<cudaStream_t>(stream)),
           "decode kernel");
    return EXL3CU_OK;
}

int exl3cu_hadamard128(float * d_values, size_t count, void * stream) {
    if (count % 128) return fail(EXL3CU_INVALID_ARGUMENT, "H128 length must be a multiple of 128");
    if (!count) return EXL3CU_OK;
    int dev, rc;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = check_device_ptr(d_values, dev, "values"))) return rc;
    if (reinterpret_cast<uintptr_t>(d_values) % 16) return fail(EXL3CU_INVALID_ARGUMENT, "values must be 16-byte aligned");
    CU_TRY(launch_hadamard128(d_values, count, static_cast<cudaStream_t>(stream)), "hadamard kernel");
    return EXL3CU_OK;
}

int exl3cu_reconstruct(const uint16_t * d_packed, const uint16_t * d_suh, const uint16_t * d_svh, size_t k,
                       size_t n, size_t first_column, size_t column_count, unsigned bits, unsigned codebook,
                       uint16_t * d_out, void * stream) {
    if (!valid_shape(k, n, 128)) return fail(EXL3CU_INVALID_ARGUMENT, "Invalid EXL3 matrix dimensions");
    if (first_column % 128 || column_count % 128)
        return fail(EXL3CU_INVALID_ARGUMENT, "H128 slices must align to 128 columns");
    int rc = exl3cu_decode_inner(d_packed, k, n, first_column, column_count, bits, codebook, d_out, stream);
    if (rc) return rc;
    int dev;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = check_device_ptr(d_suh, dev, "suh"))) return rc;
    if ((rc = check_device_ptr(d_svh, dev, "svh"))) return rc;
    CU_TRY(launch_reconstruct_blocks(d_out, k, column_count, first_column, d_suh, d_svh,
                                     static_cast<cudaStream_t>(stream)),
           "reconstruct kernel");
    return EXL3CU_OK;
}

int exl3cu_weight_from_records(const void * records, size_t record_bytes, size_t k, size_t n, unsigned bits,
                               unsigned codebook, size_t first_block, size_t block_count, int device,
                               exl3cu_weight ** out) {
    if (!records) return fail(EXL3CU_INVALID_ARGUMENT, "records is NULL");
    if (!valid_shape(k, n, 128) || bits < 1 || bits > 8)
        return fail(EXL3CU_INVALID_ARGUMENT, "k, n must be multiples of 128 and bits 1..8");
    const size_t group_bytes = 2048u * bits + 512u;
    if ((k / 128) * (n / 128) * group_bytes > record_bytes)
        return fail(EXL3CU_INVALID_ARGUMENT, "record buffer holds %zu bytes, need %zu", record_bytes,
                    (k / 128) * (n / 128) * group_bytes);
    DeviceGuard guard(device);
    if (!guard.ok) return fail(EXL3CU_INVALID_ARGUMENT, "cannot select device %d", device);
    exl3cu_weight * w = nullptr;
    int rc = make_weight(k, n, bits, codebook, first_block, block_count, device, out, &w);
    if (rc) return rc;
    // stage only the records of the selected column blocks (contiguous: nb-major)
    const size_t kb_count = k / 128;
    const size_t span = w->nblocks * kb_count * group_bytes;
    const uint8_t * src = static_cast<const uint8_t *>(records) + w->first_block * kb_count * group_bytes;
    uint8_t * staged = nullptr;
    cudaError_t e = cudaMalloc(&staged, span);
    if (e == cudaSuccess) e = cudaMemcpy(staged, src, span, cudaMemcpyDefault);
    if (e == cudaSuccess) e = launch_records_to_lsc(staged, k, bits, 0, w->nblocks, w->lsc, nullptr);
    // su from records (0..kb) of the first staged block, sv from record (nb, 0) of each block
    if (e == cudaSuccess)
        e = cudaMemcpy2D(w->su, 256, staged + 2048u * bits, group_bytes, 256, kb_count, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy2D(w->sv, 256, staged + 2048u * bits + 256u, kb_count * group_bytes, 256, w->nblocks,
                         cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(staged);
    if (e != cudaSuccess) {
        release(w);
        return cuda_fail(e, "uploading EXL3 records");
    }
    *out = w;
    return EXL3CU_OK;
}

int exl3cu_weight_from_trellis(const uint16_t * trellis, const uint16_t * suh, const uint16_t * svh, size_t k,
                               size_t n, unsigned bits, unsigned codebook, size_t first_block, size_t block_count,
                               int device, exl3cu_weight ** out) {
    if (!trellis || !suh || !svh) return fail(EXL3CU_INVALID_ARGUMENT, "trellis, suh and svh are required");
    DeviceGuard guard(device);
    if (!guard.ok) return fail(EXL3CU_INVALID_ARGUMENT, "cannot select device %d", device);
    exl3cu_weight * w = nullptr;
    int rc = make_weight(k, n, bits, codebook, first_block, block_count, device, out, &w);
    if (rc) return rc;
    const size_t tbytes = k * n * bits / 8;
    uint16_t * staged = nullptr;
    cudaError_t e = cudaMalloc(&staged, tbytes);
    if (e == cudaSuccess) e = cudaMemcpy(staged, trellis, tbytes, cudaMemcpyDefault);
    if (e == cudaSuccess) e = launch_trellis_to_lsc(staged, k, n, bits, w->first_block, w->nblocks, w->lsc, nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(w->su, suh, k * 2, cudaMemcpyDefault);
    if (e == cudaSuccess) e = cudaMemcpy(w->sv, svh + w->first_block * 128, w->nblocks * 256, cudaMemcpyDefault);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(staged);
    if (e != cudaSuccess) {
        release(w);
        return cuda_fail(e, "uploading EXL3 trellis");
    }
    *out = w;
    return EXL3CU_OK;
}

int exl3cu_weight_free(exl3cu_weight * w) {
    if (w && w->model_owned) return fail(EXL3CU_INVALID_ARGUMENT, "this weight belongs to a model handle; free the model");
    release(w);
    return EXL3CU_OK;
}

int exl3cu_weight_info(const exl3cu_weight * w, size_t * k, size_t * n_local, unsigned * bits, unsigned * codebook,
                       size_t * device_bytes) {
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    if (k) *k = w->k;
    if (n_local) *n_local = w->nblocks * 128;
    if (bits) *bits = w->bits;
    if (codebook) *codebook = w->codebook;
    if (device_bytes)
        *device_bytes = w->nblocks * (w->k / 16) * 256u * w->bits + w->k * 2 + w->nblocks * 256 + w->ws_bytes;
    return EXL3CU_OK;
}

int exl3cu_weight_decode_inner(const exl3cu_weight * w, uint16_t * d_out, void * stream) {
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    int rc = check_device_ptr(d_out, w->device, "out");
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(d_out) % 16) return fail(EXL3CU_INVALID_ARGUMENT, "out must be 16-byte aligned");
    DeviceGuard guard(w->device);
    CU_TRY(launch_lsc_decode(w->lsc, w->k, w->nblocks, w->bits, w->codebook, d_out, static_cast<cudaStream_t>(stream)),
           "device-layout decode kernel");
    return EXL3CU_OK;
}

size_t exl3cu_mul_mat_workspace_bytes(const exl3cu_weight * w) { return w ? w->ws_bytes : 0; }

int exl3cu_gemm_config(size_t min_rows, int tokens_per_cta, int splits) {
    if (tokens_per_cta < 0 || tokens_per_cta > 256 || tokens_per_cta % 32)
        return fail(EXL3CU_INVALID_ARGUMENT, "tokens_per_cta must be 0 or a multiple of 32 up to 256");
    if (splits < 0 || splits > 16 || (splits & (splits - 1)))
        return fail(EXL3CU_INVALID_ARGUMENT, "splits must be 0 or a power of two up to 16");
    if (min_rows) g_gemm_min_rows.store(min_rows, std::memory_order_relaxed);
    g_gemm_tokens.store(tokens_per_cta, std::memory_order_relaxed);
    g_gemm_splits.store(splits, std::memory_order_relaxed);
    return EXL3CU_OK;
}

int exl3cu_device_status(int device, unsigned * status, int clear) {
    if (!status) return fail(EXL3CU_INVALID_ARGUMENT, "status is NULL");
    DeviceGuard guard(device);
    if (!guard.ok) return fail(EXL3CU_INVALID_ARGUMENT, "cannot select device %d", device);
    CU_TRY(cudaDeviceSynchronize(), "synchronising before reading the device status");
    unsigned gemv = 0, gemm = 0, rows = 0, peers = 0;
    CU_TRY(peer_read_status(&peers, clear != 0), "reading the peer-exchange status word");
    CU_TRY(mul1_read_status(&gemv, clear != 0), "reading the GEMV status word");
    CU_TRY(gemm_read_status(&gemm, clear != 0), "reading the GEMM status word");
    CU_TRY(rows_read_status(&rows, clear != 0), "reading the get_rows status word");
    *status = gemv | gemm | rows | peers;
    return EXL3CU_OK;
}

int exl3cu_mul_mat(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows, size_t x_row_stride,
                   float * d_y, size_t y_row_stride, void * stream) {
    int rc = validate_mm(w, d_x, x_dtype, rows, x_row_stride, d_y, y_row_stride);
    if (rc) return rc;
    if ((rc = check_device_ptr(d_x, w->device, "x"))) return rc;
    if ((rc = check_device_ptr(d_y, w->device, "y"))) return rc;
    const MmItem item{w, d_x, x_dtype, rows, x_row_stride, d_y, y_row_stride};
    return run_cluster(&item, 1, static_cast<cudaStream_t>(stream));
}

int exl3cu_mul_mat_batch(size_t count, const exl3cu_weight * const * weights, const void * const * d_x,
                         const int * x_dtype, const size_t * rows, const size_t * x_row_stride, float * const * d_y,
                         const size_t * y_row_stride, void * stream) {
    if (!count) return EXL3CU_OK;
    if (!weights || !d_x || !x_dtype || !rows || !x_row_stride || !d_y || !y_row_stride)
        return fail(EXL3CU_INVALID_ARGUMENT, "batch arrays must not be NULL");
    std::vector<MmItem> items(count);
    for (size_t i = 0; i < count; ++i) {
        int rc = validate_mm(weights[i], d_x[i], x_dtype[i], rows[i], x_row_stride[i], d_y[i], y_row_stride[i]);
        if (!rc) rc = check_device_ptr(d_x[i], weights[i]->device, "x");
        if (!rc) rc = check_device_ptr(d_y[i], weights[i]->device, "y");
        if (rc) {
            std::string why = g_last_error;
            return fail(rc, "batch item %zu: %s", i, why.c_str());
        }
        items[i] = MmItem{weights[i], d_x[i], x_dtype[i], rows[i], x_row_stride[i], d_y[i], y_row_stride[i]};
    }
    return run_cluster(items.data(), count, static_cast<cudaStream_t>(stream));
}

int exl3cu_mul_mat_batch_ex(size_t count, const exl3cu_weight * const * weights, const void * const * d_x,
                            const int * x_form, const size_t * rows, const size_t * x_row_stride,
                            const float * const * d_norm_w, float eps, float * const * d_y,
                            const size_t * y_row_stride, const int * y_accumulate,
                            const float * const * d_x_sumsq, float * const * d_y_sumsq, void * stream) {
    if (!count) return EXL3CU_OK;
    if (!weights || !d_x || !x_form || !rows || !x_row_stride || !d_y || !y_row_stride)
        return fail(EXL3CU_INVALID_ARGUMENT, "batch arrays must not be NULL");
    std::vector<MmItem> items(count);
    for (size_t i = 0; i < count; ++i) {
        const int form = x_form[i];
        if (form < EXL3CU_F32 || form > EXL3CU_X_RMSNORM)
            return fail(EXL3CU_INVALID_ARGUMENT, "batch item %zu: unknown input form %d", i, form);
        const int dtype = form == EXL3CU_F16 ? EXL3CU_F16 : EXL3CU_F32;
        int rc = validate_mm(weights[i], d_x[i], dtype, rows[i], x_row_stride[i], d_y[i], y_row_stride[i]);
        if (!rc) rc = check_device_ptr(d_x[i], weights[i]->device, "x");
        if (!rc) rc = check_device_ptr(d_y[i], weights[i]->device, "y");
        if (!rc && form == EXL3CU_X_GLU && x_row_stride[i] < 2 * weights[i]->k)
            rc = fail(EXL3CU_INVALID_ARGUMENT, "GLU rows hold gate and up: stride at least 2k");
        if (!rc && form == EXL3CU_X_RMSNORM) {
            if (!d_norm_w || !d_norm_w[i]) rc = fail(EXL3CU_INVALID_ARGUMENT, "RMSNorm input needs norm weights");
            else if (reinterpret_cast<uintptr_t>(d_norm_w[i]) % 16)
                rc = fail(EXL3CU_INVALID_ARGUMENT, "norm weights must be 16-byte aligned");
            else rc = check_device_ptr(d_norm_w[i], weights[i]->device, "norm weights");
        }
        if (!rc && d_x_sumsq && d_x_sumsq[i]) {
            if (form != EXL3CU_X_RMSNORM) rc = fail(EXL3CU_INVALID_ARGUMENT, "x sums of squares need the RMSNorm form");
            else rc = check_device_ptr(d_x_sumsq[i], weights[i]->device, "x sums of squares");
        }
        if (!rc && d_y_sumsq && d_y_sumsq[i]) rc = check_device_ptr(d_y_sumsq[i], weights[i]->device, "y sums of squares");
        if (rc) {
            std::string why = g_last_error;
            return fail(rc, "batch item %zu: %s", i, why.c_str());
        }
        MmItem it{weights[i], d_x[i], dtype, rows[i], x_row_stride[i], d_y[i], y_row_stride[i]};
        it.x_mode = form == EXL3CU_X_GLU ? kXGlu : form == EXL3CU_X_RMSNORM ? kXRmsNorm : kXPlain;
        it.nw = form == EXL3CU_X_RMSNORM ? d_norm_w[i] : nullptr;
        it.eps = eps;
        it.y_accum = y_accumulate ? (y_accumulate[i] != 0) : 0;
        it.x_ss = d_x_sumsq ? d_x_sumsq[i] : nullptr;
        it.y_ss = d_y_sumsq ? d_y_sumsq[i] : nullptr;
        items[i] = it;
    }
    return run_cluster(items.data(), count, static_cast<cudaStream_t>(stream));
}

int exl3cu_pack_ragged(size_t n_seq, const int32_t * d_want, const int32_t * d_pos, int32_t max_rows,
                       int32_t * d_row_offsets, int32_t * d_row_seq, int32_t * d_row_pos, void * stream) {
    if (n_seq == 0 || n_seq > kMaxRaggedSeqs)
        return fail(EXL3CU_INVALID_ARGUMENT, "n_seq must be 1..%zu", kMaxRaggedSeqs);
    if (max_rows < 1 || max_rows > kMaxRaggedRows)
        return fail(EXL3CU_INVALID_ARGUMENT, "max_rows must be 1..%d", kMaxRaggedRows);
    int dev = 0, rc;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = check_device_ptr(d_want, dev, "want"))) return rc;
    if ((rc = check_device_ptr(d_pos, dev, "pos"))) return rc;
    if ((rc = check_device_ptr(d_row_offsets, dev, "row_offsets"))) return rc;
    if ((rc = check_device_ptr(d_row_seq, dev, "row_seq"))) return rc;
    if ((rc = check_device_ptr(d_row_pos, dev, "row_pos"))) return rc;
    CU_TRY(launch_pack_ragged(int(n_seq), d_want, d_pos, max_rows, d_row_offsets, d_row_seq, d_row_pos,
                              static_cast<cudaStream_t>(stream)),
           "launching the ragged batch packer");
    return EXL3CU_OK;
}

int exl3cu_mul_mat_ragged(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t x_row_stride,
                          const int32_t * d_row_offsets, size_t n_seq, size_t max_rows, float * d_y,
                          size_t y_row_stride, void * stream) {
    int rc = validate_mm(w, d_x, x_dtype, max_rows, x_row_stride, d_y, y_row_stride);
    if (rc) return rc;
    if (n_seq == 0 || n_seq > kMaxRaggedSeqs)
        return fail(EXL3CU_INVALID_ARGUMENT, "n_seq must be 1..%zu", kMaxRaggedSeqs);
    if (max_rows > size_t(kMaxRaggedRows)) return fail(EXL3CU_INVALID_ARGUMENT, "max_rows above %d", kMaxRaggedRows);
    if ((rc = check_device_ptr(d_x, w->device, "x"))) return rc;
    if ((rc = check_device_ptr(d_y, w->device, "y"))) return rc;
    if ((rc = check_device_ptr(d_row_offsets, w->device, "row_offsets"))) return rc;
    const MmItem item{w, d_x, x_dtype, max_rows, x_row_stride, d_y, y_row_stride};
    return run_gemm(item, static_cast<cudaStream_t>(stream), d_row_offsets + n_seq);
}

int exl3cu_mul_mat_ws(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows, size_t x_row_stride,
                      float * d_y, size_t y_row_stride, void * d_workspace, size_t workspace_bytes, void * stream) {
    int rc = validate_mm(w, d_x, x_dtype, rows, x_row_stride, d_y, y_row_stride);
    if (rc) return rc;
    if (workspace_bytes < w->ws_bytes)
        return fail(EXL3CU_INVALID_ARGUMENT, "workspace of %zu bytes, need %zu", workspace_bytes, w->ws_bytes);
    if (w->ws_bytes) {
        if ((rc = check_device_ptr(d_workspace, w->device, "workspace"))) return rc;
        if (reinterpret_cast<uintptr_t>(d_workspace) % 16)
            return fail(EXL3CU_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
    }
    if ((rc = check_device_ptr(d_x, w->device, "x"))) return rc;
    if ((rc = check_device_ptr(d_y, w->device, "y"))) return rc;
    DeviceGuard guard(w->device);
    return run_mm(w, d_x, x_dtype, rows, x_row_stride, d_y, y_row_stride, d_workspace,
                  static_cast<cudaStream_t>(stream));
}

int exl3cu_get_rows(const exl3cu_weight * w, const int32_t * d_ids, size_t count, float * d_out,
                    size_t out_row_stride, void * stream) {
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    if (!count) return EXL3CU_OK;
    if (count > kMaxGetRows) return fail(EXL3CU_INVALID_ARGUMENT, "count above %zu", kMaxGetRows);
    if (!d_ids || !d_out) return fail(EXL3CU_INVALID_ARGUMENT, "ids and out are required");
    if (out_row_stride < w->k) return fail(EXL3CU_INVALID_ARGUMENT, "out row stride shorter than k");
    int rc;
    if ((rc = check_device_ptr(d_ids, w->device, "ids"))) return rc;
    if ((rc = check_device_ptr(d_out, w->device, "out"))) return rc;
    DeviceGuard guard(w->device);
    CU_TRY(launch_get_rows(w->lsc, reinterpret_cast<const uint16_t *>(w->su), reinterpret_cast<const uint16_t *>(w->sv),
                           w->k, w->nblocks * 128, w->bits, w->codebook, d_ids, count, d_out, out_row_stride, false,
                           static_cast<cudaStream_t>(stream)),
           "launching get_rows");
    return EXL3CU_OK;
}

int exl3cu_get_rows_host(exl3cu_weight * w, const int32_t * h_ids, size_t count, float * h_out,
                         size_t out_row_stride, int synchronize, void * stream) {
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    if (!count) return EXL3CU_OK;
    if (count > kMaxGetRows) return fail(EXL3CU_INVALID_ARGUMENT, "count above %zu", kMaxGetRows);
    if (!h_ids || !h_out) return fail(EXL3CU_INVALID_ARGUMENT, "ids and out are required");
    if (out_row_stride < w->k) return fail(EXL3CU_INVALID_ARGUMENT, "out row stride shorter than k");
    const size_t ncols = w->nblocks * 128;
    for (size_t i = 0; i < count; ++i)
        if (h_ids[i] < 0 || size_t(h_ids[i]) >= ncols)
            return fail(EXL3CU_INVALID_ARGUMENT, "id %d at %zu outside 0..%zu", int(h_ids[i]), i, ncols - 1);
    DeviceGuard guard(w->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t ib = (count * sizeof(int32_t) + 255) & ~size_t(255), ob = count * w->k * sizeof(float);
    int rc;
    if ((rc = grow_stage(w, &w->stage_x, &w->stage_x_bytes, ib))) return rc;
    if ((rc = grow_stage(w, reinterpret_cast<void **>(&w->stage_y), &w->stage_y_bytes, ob))) return rc;
    CU_TRY(cudaMemcpyAsync(w->stage_x, h_ids, count * sizeof(int32_t), cudaMemcpyHostToDevice, st),
           "copying ids to the device");
    CU_TRY(launch_get_rows(w->lsc, reinterpret_cast<const uint16_t *>(w->su), reinterpret_cast<const uint16_t *>(w->sv),
                           w->k, ncols, w->bits, w->codebook, static_cast<const int32_t *>(w->stage_x), count,
                           w->stage_y, w->k, false, st),
           "launching get_rows");
    CU_TRY(cudaMemcpy2DAsync(h_out, out_row_stride * sizeof(float), w->stage_y, w->k * sizeof(float),
                             w->k * sizeof(float), count, cudaMemcpyDeviceToHost, st),
           "copying rows to the host");
    if (synchronize) CU_TRY(cudaStreamSynchronize(st), "synchronising the stream");
    return EXL3CU_OK;
}

int exl3cu_mul_mat_host(exl3cu_weight * w, const void * h_x, int x_dtype, size_t rows, size_t x_row_stride,
                        float * h_y, size_t y_row_stride, int synchronize, void * stream) {
    if (!h_x || !h_y) return fail(EXL3CU_INVALID_ARGUMENT, "x and y are required");
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    if (x_dtype != EXL3CU_F32 && x_dtype != EXL3CU_F16)
        return fail(EXL3CU_INVALID_ARGUMENT, "x dtype must be F32 (0) or F16 (1)");
    if (!rows) return fail(EXL3CU_INVALID_ARGUMENT, "rows must be >= 1");
    const size_t n_local = w->nblocks * 128;
    if (x_row_stride < w->k || y_row_stride < n_local)
        return fail(EXL3CU_INVALID_ARGUMENT, "row stride shorter than a row");
    DeviceGuard guard(w->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t es = x_dtype == EXL3CU_F32 ? 4 : 2;
    const size_t xb = rows * w->k * es, yb = rows * n_local * sizeof(float);
    int rc;
    if (synchronize && rows <= kZeroCopyRows) {
        // Zero-copy: x is packed into mapped pinned memory the kernel reads over the bus, y is written
        // there by the kernel's epilogue, and the host copies it out after the synchronisation.  Saves
        // the two staged copies of pageable memory (about 20 us of a decode-sized call).
        if (w->pin_x_bytes < xb || w->pin_y_bytes < yb) {
            if ((rc = grow_pinned(&w->pin_x, &w->pin_x_bytes, xb))) return rc;
            if ((rc = grow_pinned(reinterpret_cast<void **>(&w->pin_y), &w->pin_y_bytes, yb))) return rc;
            CU_TRY(cudaHostGetDevicePointer(&w->pin_x_dev, w->pin_x, 0), "mapping pinned x");
            CU_TRY(cudaHostGetDevicePointer(reinterpret_cast<void **>(&w->pin_y_dev), w->pin_y, 0), "mapping pinned y");
        }
        for (size_t r = 0; r < rows; ++r)
            std::memcpy(static_cast<char *>(w->pin_x) + r * w->k * es,
                        static_cast<const char *>(h_x) + r * x_row_stride * es, w->k * es);
        const MmItem item{w, w->pin_x_dev, x_dtype, rows, w->k, w->pin_y_dev, n_local};
        if ((rc = run_cluster(&item, 1, st))) return rc;
        CU_TRY(cudaStreamSynchronize(st), "synchronising the stream");
        for (size_t r = 0; r < rows; ++r)
            std::memcpy(h_y + r * y_row_stride, w->pin_y + r * n_local, n_local * sizeof(float));
        return EXL3CU_OK;
    }
    if ((rc = grow_stage(w, &w->stage_x, &w->stage_x_bytes, xb))) return rc;
    if ((rc = grow_stage(w, reinterpret_cast<void **>(&w->stage_y), &w->stage_y_bytes, yb))) return rc;
    CU_TRY(cudaMemcpy2DAsync(w->stage_x, w->k * es, h_x, x_row_stride * es, w->k * es, rows, cudaMemcpyHostToDevice, st),
           "copying x to the device");
    const MmItem item{w, w->stage_x, x_dtype, rows, w->k, w->stage_y, n_local};
    rc = run_cluster(&item, 1, st);
    if (rc) return rc;
    CU_TRY(cudaMemcpy2DAsync(h_y, y_row_stride * sizeof(float), w->stage_y, n_local * sizeof(float),
                             n_local * sizeof(float), rows, cudaMemcpyDeviceToHost, st),
           "copying y to the host");
    if (synchronize) CU_TRY(cudaStreamSynchronize(st), "synchronising the stream");
    return EXL3CU_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free operator entry.
//
// Some callers may not call cudaMalloc/cudaFree at all: a host framework that
// owns and budgets every byte of device memory and plans its buffers before it
// runs (ggml's backend scheduler works this way), or a latency-critical loop
// that cannot afford the device-wide synchronisation cudaFree implies.  For
// them, exl3cu_mul_mat_noalloc runs the split-K GEMV with its partial sums and
// arrival tickets in the file-scope array below instead of a handle- or
// caller-owned workspace.
//
// * Size: kStaticScratchBytes (4 MiB), held by every GPU that loads this
//   library until the process exits.  A handle whose split-K plan needs more is
//   rejected with EXL3CU_NO_SUPPORT and a message naming both sizes.
// * Host code sees only a host-side stand-in for the array, so its device
//   address is fetched with cudaGetSymbolAddress, once per device, with that
//   device current -- done by the first call on each device, which should
//   therefore come before any stream capture.
// * Every call shares the array and it keeps the previous call's contents: each
//   call clears the ticket counters it uses (cudaMemsetAsync on the caller's
//   stream) before launching.  Calls whose executions overlap on the GPU -- on
//   different streams, or from different threads without ordering -- race on
//   the array and give wrong results; order them on one stream.
// * Nothing here allocates: no cudaMalloc, cudaFree or allocating library call.
// ---------------------------------------------------------------------------

namespace {
constexpr size_t kStaticScratchBytes = size_t(4) << 20;
}

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace {

std::mutex g_static_scratch_mu;
void * g_static_scratch_dev[64] = {};

// Device address of g_static_scratch on `device` (current on entry).
int static_scratch_address(int device, void ** out) {
    if (device < 0 || device >= 64) return fail(EXL3CU_NO_SUPPORT, "device index %d beyond 63", device);
    std::lock_guard<std::mutex> lock(g_static_scratch_mu);
    if (!g_static_scratch_dev[device]) {
        void * p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
        g_static_scratch_dev[device] = p;
    }
    *out = g_static_scratch_dev[device];
    return EXL3CU_OK;
}

}  // namespace

extern "C" int exl3cu_mul_mat_noalloc(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows,
                                      size_t x_row_stride, float * d_y, size_t y_row_stride, void * stream) {
    int rc = validate_mm(w, d_x, x_dtype, rows, x_row_stride, d_y, y_row_stride);
    if (rc) return rc;
    if ((rc = check_device_ptr(d_x, w->device, "x"))) return rc;
    if ((rc = check_device_ptr(d_y, w->device, "y"))) return rc;
    if (w->ws_bytes > kStaticScratchBytes)
        return fail(EXL3CU_NO_SUPPORT, "this weight's split-K plan needs %zu bytes of scratch; the static scratch holds %zu",
                    w->ws_bytes, kStaticScratchBytes);
    DeviceGuard guard(w->device);
    if (!guard.ok) return fail(EXL3CU_CUDA_ERROR, "cannot select device %d", w->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void * scratch = nullptr;
    if (w->ws_bytes) {
        if ((rc = static_scratch_address(w->device, &scratch))) return rc;
        // tickets follow the partials (run_mm's workspace layout) and must start at zero
        const size_t partial_bytes = w->nblocks * size_t(w->plan.splits) * 8 * 128 * sizeof(float);
        CU_TRY(cudaMemsetAsync(static_cast<char *>(scratch) + partial_bytes, 0, w->nblocks * sizeof(unsigned), st),
               "clearing the static scratch tickets");
    }
    return run_mm(w, d_x, x_dtype, rows, x_row_stride, d_y, y_row_stride, scratch, st);
}

// ---------------------------------------------------------------------------
// The operator of one rank of a column split, with its all-gather: y = x . W_local stored into
// every rank's y buffer over NVLink (half (E & 1) for this rank's E-th call), then the epoch
// published to every rank.  1..4 rows of mul1 weights: one launch, the GEMV's epilogue storing to
// the peers.  Otherwise the operator writes d_slice and exl3cu_store_peers sends it.
extern "C" int exl3cu_mul_mat_peers(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows,
                                    size_t x_row_stride, float * d_slice, size_t slice_stride, int npeers,
                                    void * const * d_y_peers, size_t y_row_stride, size_t y_half, size_t y_col0,
                                    const unsigned * d_state, void * stream) {
    if (npeers < 1 || npeers > kMaxPeers) return fail(EXL3CU_INVALID_ARGUMENT, "mul_mat_peers: 1..%d ranks", kMaxPeers);
    if (!d_y_peers || !d_state) return fail(EXL3CU_INVALID_ARGUMENT, "mul_mat_peers: NULL peer arrays or state");
    {
        const int rc = check_device_ptr(d_state, -1, "state");
        if (rc) return rc;
    }
    if (y_row_stride % 4 || y_half % 4 || y_col0 % 4)
        return fail(EXL3CU_INVALID_ARGUMENT, "mul_mat_peers: y strides and offsets must be multiples of 4 words");
    if (!w) return fail(EXL3CU_INVALID_ARGUMENT, "weight handle is NULL");
    const size_t n_local = w->nblocks * 128;
    if (y_row_stride < y_col0 + n_local || y_half < rows * y_row_stride)
        return fail(EXL3CU_INVALID_ARGUMENT, "mul_mat_peers: the slice does not fit the peers' y buffers");
    PeerOut po{};
    for (int p = 0; p < npeers; ++p) {
        const int rc = check_device_ptr(d_y_peers[p], -1, "a peer's y buffer");  // IPC mappings: any device
        if (rc) return rc;
        po.y[p] = static_cast<unsigned long long *>(d_y_peers[p]);
    }
    po.own_state = d_state;
    po.y_stride = (long long)y_row_stride;
    po.y_half = (long long)y_half;
    po.y_col0 = (long long)y_col0;
    po.npeers = npeers;
    const bool gemv = w->codebook == EXL3CU_CB_MUL1 && rows >= 1 && rows < gemm_min_rows() &&
                      mul1_supported(w->bits, int(rows < 64 ? rows : 64));
    const bool gemm = w->codebook == EXL3CU_CB_MUL1 && rows >= gemm_min_rows() && rows <= kGemmRowsPerLaunch;
    if (gemm) {  // one tcgen05 GEMM launch pair whose epilogue stores to the peers
        float * y_unused = d_slice ? d_slice : reinterpret_cast<float *>(po.y[0]);
        int rc = validate_mm(w, d_x, x_dtype, rows, x_row_stride, y_unused, n_local);
        if (rc) return rc;
        if ((rc = check_device_ptr(d_x, w->device, "x"))) return rc;
        const MmItem item{w, d_x, x_dtype, rows, x_row_stride, y_unused, n_local};
        return run_gemm(item, static_cast<cudaStream_t>(stream), nullptr, &po);
    }
    if (gemv) {
        // the operator's own y argument is not written on this path: validate shapes against the slice
        float * y_unused = d_slice;
        if (!y_unused) y_unused = reinterpret_cast<float *>(po.y[0]);
        int rc = validate_mm(w, d_x, x_dtype, rows, x_row_stride, y_unused, n_local);
        if (rc) return rc;
        if ((rc = check_device_ptr(d_x, w->device, "x"))) return rc;
        const MmItem item{w, d_x, x_dtype, rows, x_row_stride, y_unused, n_local};
        return run_cluster(&item, 1, static_cast<cudaStream_t>(stream), &po);
    }
    if (!d_slice) return fail(EXL3CU_INVALID_ARGUMENT, "mul_mat_peers: this operand needs d_slice");
    int rc = exl3cu_mul_mat(w, d_x, x_dtype, rows, x_row_stride, d_slice, slice_stride, stream);
    if (rc) return rc;
    return exl3cu_store_peers(d_slice, rows, n_local, slice_stride, npeers, d_y_peers, y_row_stride, y_half, y_col0,
                              d_state, stream);
}

// ---------------------------------------------------------------------------
// Internal hooks for the other C-ABI translation units (the model loader).
namespace exl3cu {

bool pdl_launch_enabled() { return pdl_enabled(); }

int api_fail(int status, const char * message) { return fail(status, "%s", message); }

int api_cuda_fail(cudaError_t e, const char * what) { return cuda_fail(e, what); }

int api_check_device_ptr(const void * p, int device, const char * name) { return check_device_ptr(p, device, name); }

void weight_set_model_owned(::exl3cu_weight * w) { w->model_owned = true; }

void weight_free_owned(::exl3cu_weight * w) { release(w); }

WeightGeometry weight_geometry(const ::exl3cu_weight * w) {
    return WeightGeometry{w->k,      w->nblocks * 128, w->bits, w->codebook, w->device, w->lsc,
                          reinterpret_cast<const uint16_t *>(w->su), reinterpret_cast<const uint16_t *>(w->sv)};
}

}  // namespace exl3cu
