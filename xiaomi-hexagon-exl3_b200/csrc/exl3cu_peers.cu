// Peer-memory exchange for the column-split operator (BASELINE configs[4] on
// 2..8 GPUs, one process per GPU).  It replaces the NCCL all-gather of the
// output slices: every rank stores its slice of y straight into every peer's
// y buffer over NVLink (CUDA IPC mappings, plain P2P stores), then raises the
// call's epoch in every peer's flag word; each rank's wait kernel returns once
// all ranks' flags show the epoch.  No counterpart in the reference, whose
// operator (src/exl3-ggml.cpp:51-92) splits columns over CPU threads of one
// process (`for nb = ith; nb < n/128; nb += nth`, src/exl3-ggml.cpp:74).
//
// Ordering: a rank's store kernel comes after its consumers of the previous
// output on its stream, and a peer can be at most one call ahead (its next
// store waits on this rank's flag), so y is double-buffered by epoch parity and
// flags compare modulo 2^32.  The epoch lives on the device (a counter the
// store kernel advances), so a call can be captured in a CUDA graph and
// replayed; the wait kernel copies the finished half into a fixed output.
// Every wait is bounded: after about a second it sets kStatusWaitTimeout in
// the device status and returns.  No multicast, no NVLS: P2P stores only.
#include "exl3cu.h"
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"

#include <cstring>

namespace exl3cu {

static __device__ unsigned g_peer_status;

constexpr unsigned kPeerWaitRounds = 1u << 20;  // polls of >= ~1 us: about a second

// A rank's state words (its IPC-shared flag buffer): [0, 8) every rank's last
// epoch, [8] the storing kernel's arrival ticket, [9] this rank's epoch counter.
constexpr int kTicketWord = kPeerTicketWord;
constexpr int kEpochWord = kPeerEpochWord;

struct PeerArgs {
    float * y[kMaxPeers];         // every rank's y buffer [2][rows_cap][...] (this rank's included)
    unsigned * state[kMaxPeers];  // every rank's state words
    const float * src;            // this rank's slice [rows][src_stride]
    long long src_stride;
    long long y_stride;
    long long y_half;             // floats between the two halves of a y buffer
    long long y_col0;
    int rows, cols;
    int npeers, rank;
};

// The call's epoch E = this rank's counter + 1 (on the device, so the call can be replayed from a
// CUDA graph); float4s of the slice into half (E & 1) of every rank's y; the last CTA to finish
// (ticket) publishes E in every rank's state and advances the counter.
__global__ void __launch_bounds__(256) k_store_peers(const PeerArgs a) {
    __shared__ int last;
    pdl_trigger();
    pdl_wait_primary();  // the slice is written by the previous kernel
    unsigned * own = a.state[a.rank];
    const unsigned E = *reinterpret_cast<volatile unsigned *>(own + kEpochWord) + 1u;
    const long long half = (E & 1u) ? a.y_half : 0;
    const int c4 = a.cols / 4;
    const long long total = (long long)a.rows * c4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = int(i / c4);
        const int c = int(i - (long long)r * c4) * 4;
        const float4 v = *reinterpret_cast<const float4 *>(a.src + r * a.src_stride + c);
        for (int p = 0; p < a.npeers; ++p)
            *reinterpret_cast<float4 *>(a.y[p] + half + r * a.y_stride + a.y_col0 + c) = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();  // this CTA's peer stores are visible to every GPU before its ticket
        last = atomicAdd(own + kTicketWord, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        own[kTicketWord] = 0u;   // every CTA has arrived (and read the counter): reset for the next call
        own[kEpochWord] = E;
        __threadfence_system();  // every CTA's stores are ordered before the flags
        for (int p = 0; p < a.npeers; ++p)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.state[p] + a.rank), "r"(E) : "memory");
    }
}

// Every CTA: thread 0 waits until every rank's flag has reached this rank's epoch (modulo 2^32: a
// rank may be one call ahead); then the CTA copies its share of the finished half of y into out.
__global__ void __launch_bounds__(256) k_wait_peers(const unsigned * state, int npeers, const float * y,
                                                    long long y_half, long long y_stride, float * out,
                                                    long long out_stride, int rows, int cols) {
    __shared__ unsigned epoch_s;
    pdl_trigger();
    pdl_wait_primary();  // this rank's own storing kernel has finished: only other GPUs are waited for
    if (threadIdx.x == 0) {
        const unsigned E = *reinterpret_cast<const volatile unsigned *>(state + kEpochWord);
        epoch_s = E;
        for (int p = 0; p < npeers; ++p) {
            unsigned i = 0;
            for (; i < kPeerWaitRounds; ++i) {
                unsigned v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(state + p) : "memory");
                if (int(v - E) >= 0) break;
                __nanosleep(500);
            }
            if (i == kPeerWaitRounds) {
                atomicOr(&g_peer_status, kStatusWaitTimeout);
                break;
            }
        }
    }
    __syncthreads();
    if (!out) return;
    const float * src = y + ((epoch_s & 1u) ? y_half : 0);
    const int c4 = cols / 4;
    const long long total = (long long)rows * c4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = int(i / c4);
        const int c = int(i - (long long)r * c4) * 4;
        *reinterpret_cast<float4 *>(out + r * out_stride + c) = *reinterpret_cast<const float4 *>(src + r * y_stride + c);
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
                       float * const * d_y_peers, size_t y_row_stride, size_t y_half, size_t y_col0,
                       unsigned * const * d_state_peers, int rank, void * stream) {
    if (npeers < 1 || npeers > kMaxPeers || rank < 0 || rank >= npeers)
        return api_fail(EXL3CU_INVALID_ARGUMENT, "store_peers: 1..8 ranks and 0 <= rank < npeers");
    if (!d_slice || !d_y_peers || !d_state_peers || !rows || !cols)
        return api_fail(EXL3CU_INVALID_ARGUMENT, "store_peers: NULL or empty argument");
    if (cols % 4 || slice_stride % 4 || y_row_stride % 4 || y_half % 4 || y_col0 % 4 || slice_stride < cols)
        return api_fail(EXL3CU_INVALID_ARGUMENT, "store_peers: columns, strides and offsets must be multiples of 4");
    PeerArgs a{};
    for (int p = 0; p < npeers; ++p) {
        if (!d_y_peers[p] || !d_state_peers[p]) return api_fail(EXL3CU_INVALID_ARGUMENT, "store_peers: NULL peer");
        a.y[p] = d_y_peers[p];
        a.state[p] = d_state_peers[p];
    }
    a.src = d_slice;
    a.src_stride = (long long)slice_stride;
    a.y_stride = (long long)y_row_stride;
    a.y_half = (long long)y_half;
    a.y_col0 = (long long)y_col0;
    a.rows = int(rows);
    a.cols = int(cols);
    a.npeers = npeers;
    a.rank = rank;
    const size_t f4 = rows * cols / 4;
    const unsigned grid = unsigned(f4 < 256 ? 1 : (f4 + 255) / 256 < 296 ? (f4 + 255) / 256 : 296);
    const cudaError_t e = launch_pdl(k_store_peers, grid, static_cast<cudaStream_t>(stream), a);
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "launching the peer stores");
}

int exl3cu_wait_peers(const unsigned * d_state, int npeers, const float * d_y, size_t y_row_stride, size_t y_half,
                      float * d_out, size_t out_row_stride, size_t rows, size_t cols, void * stream) {
    if (!d_state || npeers < 1 || npeers > kMaxPeers) return api_fail(EXL3CU_INVALID_ARGUMENT, "wait_peers: 1..8 ranks");
    if (d_out && (!d_y || cols % 4 || y_row_stride % 4 || y_half % 4 || out_row_stride % 4))
        return api_fail(EXL3CU_INVALID_ARGUMENT, "wait_peers: y, strides and columns must be multiples of 4 floats");
    const size_t f4 = d_out ? rows * cols / 4 : 0;
    const unsigned grid = unsigned(f4 < 256 ? 1 : (f4 + 255) / 256 < 148 ? (f4 + 255) / 256 : 148);
    const cudaError_t e = launch_pdl(k_wait_peers, grid, static_cast<cudaStream_t>(stream), d_state, npeers, d_y,
                                     (long long)y_half, (long long)y_row_stride, d_out, (long long)out_row_stride,
                                     int(rows), int(cols));
    return e == cudaSuccess ? EXL3CU_OK : api_cuda_fail(e, "launching the peer wait");
}

}  // extern "C"
