// Peer-memory exchange for the column-split operator (BASELINE configs[4] on
// 2..8 GPUs, one process per GPU).  It replaces the NCCL all-gather of the
// output slices: every rank stores its slice of y straight into every peer's
// y buffer over NVLink (CUDA IPC mappings, plain P2P stores), and every rank's
// wait kernel copies the whole row out of its own buffer once every element of
// this call has arrived.  No counterpart in the reference, whose operator
// (src/exl3-ggml.cpp:51-92) splits columns over CPU threads of one process
// (`for nb = ith; nb < n/128; nb += nth`, src/exl3-ggml.cpp:74).
//
// Protocol: self-validating pairs, no fences and no flags.  Every element of
// a y buffer is one 8-byte word (epoch << 32 | float bits), written with a
// single-copy-atomic 8-byte store, so a reader that sees a word of epoch E
// sees that call's value in the same word; the reader polls each element
// until its epoch is this call's.  (A fence and a flag per call measured
// several microseconds per launch: a system-scope fence waits for far more
// than the stores it orders.)  The epoch E = this rank's counter + 1 lives on
// the device, so calls can be captured in a CUDA graph and replayed; the wait
// kernel advances the counter.  A rank can be at most one call ahead of
// another (its next store follows its wait for this call), so y is
// double-buffered by epoch parity.  Every wait is bounded: after about a
// second it sets kStatusWaitTimeout in the device status, copies what is
// there and returns.  No multicast, no NVLS: P2P stores only.
#include "exl3cu.h"
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"

#include <cstring>

namespace exl3cu {

static __device__ unsigned g_peer_status;

constexpr unsigned kPeerWaitRounds = 1u << 24;  // polls about 64 ns apart: about a second

// A rank's state words (16, zero-initialised): [kPeerTicketWord] the wait kernel's arrival
// ticket (reset by its last CTA), [kPeerEpochWord] this rank's epoch counter (calls completed).

struct PeerArgs {
    unsigned long long * y[kMaxPeers];  // every rank's pair buffer [2][rows_cap][y_stride] (this rank's included)
    const unsigned * own_state;         // this rank's state words
    const float * src;                  // this rank's slice [rows][src_stride]
    long long src_stride;
    long long y_stride;
    long long y_half;                   // pairs between the two halves of a y buffer
    long long y_col0;
    int rows, cols;
    int npeers;
};

// The call's epoch E = this rank's counter + 1; the slice's values, as (E, value) pairs, into half
// (E & 1) of every rank's y buffer.
__global__ void __launch_bounds__(256) k_store_peers(const PeerArgs a) {
    pdl_trigger();
    pdl_wait_primary();  // the slice is written by the previous kernel
    const unsigned E = *reinterpret_cast<const volatile unsigned *>(a.own_state + kPeerEpochWord) + 1u;
    const long long half = (E & 1u) ? a.y_half : 0;
    const int c4 = a.cols / 4;
    const long long total = (long long)a.rows * c4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = int(i / c4);
        const int c = int(i - (long long)r * c4) * 4;
        const float4 v = *reinterpret_cast<const float4 *>(a.src + r * a.src_stride + c);
        const long long off = half + r * a.y_stride + a.y_col0 + c;
        for (int p = 0; p < a.npeers; ++p) store_pairs4(a.y[p] + off, v, E);
    }
}

// Every element of the call's half of this rank's y: wait (bounded) until its epoch is this call's,
// then copy its value into out; the last CTA (ticket) advances this rank's counter.  A thread that
// gives up once raises the status and stops waiting, so the whole kernel gives up in about a second.
__global__ void __launch_bounds__(256) k_wait_peers(unsigned * state, const unsigned long long * y,
                                                    long long y_half, long long y_stride, float * out,
                                                    long long out_stride, int rows, int cols) {
    __shared__ int last;
    pdl_trigger();
    pdl_wait_primary();  // this rank's own storing kernel has finished: only other GPUs are waited for
    const unsigned E = *reinterpret_cast<const volatile unsigned *>(state + kPeerEpochWord) + 1u;
    const unsigned long long * src = y + ((E & 1u) ? y_half : 0);
    const long long total = (long long)rows * cols;
    bool patient = true;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = int(i / cols);
        const int c = int(i - (long long)r * cols);
        const unsigned long long * w = src + r * y_stride + c;
        unsigned long long v = load_pair(w);
        if (unsigned(v >> 32) != E && patient) {
            unsigned n = 0;
            for (; n < kPeerWaitRounds && unsigned(v >> 32) != E; ++n) {
                __nanosleep(64);
                v = load_pair(w);
            }
            if (n == kPeerWaitRounds) {
                atomicOr(&g_peer_status, kStatusWaitTimeout);
                patient = false;
            }
        }
        if (out) out[r * out_stride + c] = __uint_as_float(unsigned(v));
    }
    if (gridDim.x == 1) {
        __syncthreads();
        if (threadIdx.x == 0) state[kPeerEpochWord] = E;
        return;
    }
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(state + kPeerTicketWord, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last && threadIdx.x == 0) {
        state[kPeerTicketWord] = 0u;  // every CTA has read the counter: reset for the next call
        state[kPeerEpochWord] = E;
    }
}

// 256-thread launch, with programmatic dependent launch when it is enabled.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = pdl_launch_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

cudaError_t peer_read_status(unsigned * out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_peer_status, sizeof(unsigned));
    if (e == cudaSuccess && clear && *out) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_peer_status, &zero, sizeof(unsigned));
    }
    return e;
}

}  // namespace exl3cu

using namespace exl3cu;

namespace {

struct Guard {
    int prev = -1;
    bool ok = false;
    explicit Guard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) return;
        ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~Guard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int exl3cu_ipc_alloc(int device, size_t bytes, void ** out_ptr, void * out_handle) {
    if (!out_ptr || !out_handle || !bytes) return api_fail(EXL3CU_INVALID_ARGUMENT, "ipc_alloc: NULL or empty");
    Guard g(device);
    if (!g.ok) return api_fail(EXL3CU_INVALID_ARGUMENT, "ipc_alloc: cannot select the device");
    void * p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return api_cuda_fail(e, "allocating a peer buffer");
    if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess) {
        cudaFree(p);
        return api_cuda_fail(e, "clearing a peer buffer");
    }
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
        cudaFree(p);
        return api_cuda_fail(e, "exporting a peer buffer");
    }
    std::memcpy(out_handle, &h, sizeof(h));
    *out_ptr = p;
    return EXL3CU_OK;
}

int exl3cu_ipc_free(int device, void * ptr) {
    Guard g(device);
    if (!g.ok) return api_fail(EXL3CU_INVALID_ARGUMENT, "ipc_free: cannot select the device");
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "freeing a peer buffer");
}

int exl3cu_ipc_open(int device, const void * handle, void ** out_ptr) {
    if (!handle || !out_ptr) return api_fail(EXL3CU_INVALID_ARGUMENT, "ipc_open: NULL argument");
    Guard g(device);
    if (!g.ok) return api_fail(EXL3CU_INVALID_ARGUMENT, "ipc_open: cannot select the device");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "mapping a peer's buffer");
}

int exl3cu_ipc_close(int device, void * ptr) {
    Guard g(device);
    if (!g.ok) return api_fail(EXL3CU_INVALID_ARGUMENT, "ipc_close: cannot select the device");
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "unmapping a peer's buffer");
}

int exl3cu_store_peers(const float * d_slice, size_t rows, size_t cols, size_t slice_stride, int npeers,
                       void * const * d_y_peers, size_t y_row_stride, size_t y_half, size_t y_col0,
                       const unsigned * d_state, void * stream) {
    if (npeers < 1 || npeers > kMaxPeers) return api_fail(EXL3CU_INVALID_ARGUMENT, "store_peers: 1..8 ranks");
    if (!d_slice || !d_y_peers || !d_state || !rows || !cols)
        return api_fail(EXL3CU_INVALID_ARGUMENT, "store_peers: NULL or empty argument");
    if (cols % 4 || slice_stride % 4 || y_row_stride % 4 || y_half % 4 || y_col0 % 4 || slice_stride < cols ||
        y_row_stride < y_col0 + cols || y_half < rows * y_row_stride)
        return api_fail(EXL3CU_INVALID_ARGUMENT,
                        "store_peers: columns, strides and offsets must be multiples of 4 and fit the buffers");
    int rc = api_check_device_ptr(d_slice, -1, "slice");
    if (!rc) rc = api_check_device_ptr(d_state, -1, "state");
    if (rc) return rc;
    PeerArgs a{};
    for (int p = 0; p < npeers; ++p) {
        if ((rc = api_check_device_ptr(d_y_peers[p], -1, "a peer's y buffer"))) return rc;  // IPC mappings: any device
        a.y[p] = static_cast<unsigned long long *>(d_y_peers[p]);
    }
    a.own_state = d_state;
    a.src = d_slice;
    a.src_stride = (long long)slice_stride;
    a.y_stride = (long long)y_row_stride;
    a.y_half = (long long)y_half;
    a.y_col0 = (long long)y_col0;
    a.rows = int(rows);
    a.cols = int(cols);
    a.npeers = npeers;
    const size_t f4 = rows * cols / 4;
    const unsigned grid = unsigned(f4 < 256 ? 1 : (f4 + 255) / 256 < 296 ? (f4 + 255) / 256 : 296);
    const cudaError_t e = launch_pdl(k_store_peers, grid, static_cast<cudaStream_t>(stream), a);
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "launching the peer stores");
}

int exl3cu_wait_peers(unsigned * d_state, const void * d_y, size_t y_row_stride, size_t y_half, float * d_out,
                      size_t out_row_stride, size_t rows, size_t cols, void * stream) {
    if (!d_state || !d_y || !rows || !cols) return api_fail(EXL3CU_INVALID_ARGUMENT, "wait_peers: NULL or empty argument");
    if (y_row_stride < cols || y_half < rows * y_row_stride || (d_out && out_row_stride < cols))
        return api_fail(EXL3CU_INVALID_ARGUMENT, "wait_peers: the rows do not fit the buffers");
    int rc = api_check_device_ptr(d_state, -1, "state");
    if (!rc) rc = api_check_device_ptr(d_y, -1, "y");
    if (!rc && d_out) rc = api_check_device_ptr(d_out, -1, "out");
    if (rc) return rc;
    const size_t n = rows * cols;
    const unsigned grid = unsigned(n <= 1024 ? 1 : (n + 1023) / 1024 < 148 ? (n + 1023) / 1024 : 148);
    const cudaError_t e =
        launch_pdl(k_wait_peers, grid, static_cast<cudaStream_t>(stream), d_state,
                   static_cast<const unsigned long long *>(d_y), (long long)y_half, (long long)y_row_stride, d_out,
                   (long long)out_row_stride, int(rows), int(cols));
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "launching the peer wait");
}

}  // extern "C"
