// exl3:: host API (include/exl3_codec.h) over the exl3cu C ABI.
//
// Same signatures, layouts and std::invalid_argument contract as the
// reference's src/exl3_codec.cpp; the work runs on the current CUDA device.
// A call stages its host buffers in a per-thread, per-device device buffer
// that only grows, runs on a per-thread stream, copies the result back and
// synchronises before returning, so nothing is allocated per call once the
// buffer has reached the working size.  decode_codebook() reads a 65536-entry
// table per (device, codebook) that the GPU codebook kernel fills on first use
// -- the reference likewise builds its state tables lazily
// (src/exl3_codec.cpp:94-100).
#include "exl3_codec.h"

#include <cuda_runtime.h>

#include <array>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "exl3cu.h"

namespace exl3 {
namespace {

void validate(unsigned bits, Codebook codebook) {
    if (bits < 1 || bits > 8) throw std::invalid_argument("EXL3 integer bitrate must be in [1,8]");
    if (static_cast<uint32_t>(codebook) > 2) throw std::invalid_argument("Unknown EXL3 codebook");
}

void validate_shape(size_t k, size_t n, size_t multiple) {
    if (!k || !n || k % multiple || n % multiple || k > std::numeric_limits<size_t>::max() / n)
        throw std::invalid_argument("Invalid EXL3 matrix dimensions");
}

void check_cuda(cudaError_t e, const char * what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void check_status(int rc) {
    if (rc == EXL3CU_INVALID_ARGUMENT) throw std::invalid_argument(exl3cu_last_error());
    if (rc) throw std::runtime_error(std::string("exl3cu: ") + exl3cu_last_error());
}

int current_device() {
    int d = 0;
    check_cuda(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}

// This thread's stream and staging buffer on one device.  The buffer grows to
// the largest call seen and is reused; a call synchronises its stream before
// returning, so no copy or kernel of an earlier call still uses it.
struct Staging {
    cudaStream_t stream = nullptr;
    char * buf = nullptr;
    size_t cap = 0;
    Staging() { check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate"); }
    ~Staging() {
        if (buf) cudaFree(buf);
        if (stream) cudaStreamDestroy(stream);
    }
    Staging(const Staging &) = delete;
    Staging & operator=(const Staging &) = delete;
    // `parts` byte counts, each region 256-byte aligned; returns their device addresses.
    template <size_t N>
    std::array<char *, N> carve(const std::array<size_t, N> & parts) {
        size_t total = 0;
        for (size_t b : parts) total += (b + 255) & ~size_t(255);
        if (total > cap) {
            if (buf) check_cuda(cudaFree(buf), "cudaFree");
            buf = nullptr;
            cap = 0;
            check_cuda(cudaMalloc(&buf, total), "cudaMalloc");
            cap = total;
        }
        std::array<char *, N> out{};
        size_t off = 0;
        for (size_t i = 0; i < N; ++i) {
            out[i] = buf + off;
            off += (parts[i] + 255) & ~size_t(255);
        }
        return out;
    }
    void upload(void * dst, const void * src, size_t bytes) {
        check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream), "copy to device");
    }
    void download(void * dst, const void * src, size_t bytes) {
        check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream), "copy to host");
    }
    void sync() { check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize"); }
};

Staging & staging() {
    thread_local std::map<int, std::unique_ptr<Staging>> per_device;
    auto & slot = per_device[current_device()];
    if (!slot) slot.reset(new Staging());
    return *slot;
}

}  // namespace

float half_to_float(uint16_t value) {
    const uint32_t sign = uint32_t(value >> 15) << 31;
    const uint32_t exp5 = (value >> 10) & 0x1fu;
    const uint32_t mant = value & 0x3ffu;
    uint32_t bits;
    if (exp5 == 0) {
        if (!mant) {
            bits = sign;
        } else {  // subnormal: normalise the mantissa into an fp32 normal
            int shift = 0;
            uint32_t m = mant;
            while (!(m & 0x400u)) { m <<= 1; ++shift; }
            bits = sign | (uint32_t(113 - shift) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (exp5 == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp5 + 112u) << 23) | (mant << 13);
    }
    float out;
    std::memcpy(&out, &bits, sizeof(out));
    return out;
}

uint16_t float_to_half(float value) {
    uint32_t bits;
    std::memcpy(&bits, &value, sizeof(bits));
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const uint32_t exp8 = (bits >> 23) & 0xffu;
    const uint32_t mant = bits & 0x7fffffu;
    auto rne = [](uint32_t v, unsigned sh) {
        const uint32_t keep = v >> sh, rest = v & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        return keep + ((rest > half) || (rest == half && (keep & 1u)));
    };
    if (exp8 == 0xffu) return uint16_t(sign | (mant ? 0x7e00u : 0x7c00u));
    if (exp8 >= 143u) return uint16_t(sign | 0x7c00u);
    if (exp8 <= 101u) return uint16_t(sign);
    if (exp8 <= 112u) return uint16_t(sign | rne(mant | 0x800000u, 126u - exp8));
    return uint16_t(sign | (((exp8 - 112u) << 10) + rne(mant, 13u)));
}

uint16_t decode_codebook(uint16_t state, Codebook codebook) {
    if (static_cast<uint32_t>(codebook) > 2) throw std::invalid_argument("Unknown EXL3 codebook");
    static std::mutex mu;
    static std::map<std::pair<int, uint32_t>, std::vector<uint16_t>> tables;
    const auto key = std::make_pair(current_device(), static_cast<uint32_t>(codebook));
    std::lock_guard<std::mutex> g(mu);
    auto it = tables.find(key);
    if (it == tables.end()) {
        // every state once through the device codebook kernel
        std::vector<uint16_t> states(65536), table(65536);
        for (size_t i = 0; i < states.size(); ++i) states[i] = uint16_t(i);
        Staging & st = staging();
        const auto d = st.carve(std::array<size_t, 2>{65536 * 2, 65536 * 2});
        st.upload(d[0], states.data(), 65536 * 2);
        check_status(exl3cu_decode_codebook(reinterpret_cast<const uint16_t *>(d[0]), 65536,
                                            static_cast<unsigned>(codebook), reinterpret_cast<uint16_t *>(d[1]),
                                            st.stream));
        st.download(table.data(), d[1], 65536 * 2);
        st.sync();
        it = tables.emplace(key, std::move(table)).first;
    }
    return it->second[state];
}

void decode_tile(const uint16_t * packed, unsigned bits, Codebook codebook, uint16_t * row_major) {
    validate(bits, codebook);
    decode_inner(packed, 16, 16, bits, codebook, row_major);
}

void decode_inner(const uint16_t * packed, size_t k, size_t n, unsigned bits, Codebook codebook, uint16_t * output) {
    decode_inner_slice(packed, k, n, 0, n, bits, codebook, output);
}

void decode_inner_slice(const uint16_t * packed, size_t k, size_t n, size_t first_column, size_t column_count,
                        unsigned bits, Codebook codebook, uint16_t * output) {
    validate(bits, codebook);
    validate_shape(k, n, 16);
    if (!column_count || first_column % 16 || column_count % 16 || first_column > n ||
        column_count > n - first_column)
        throw std::invalid_argument("Invalid EXL3 column slice");
    const size_t packed_bytes = k * n * bits / 8;
    const size_t out_bytes = k * column_count * 2;
    Staging & st = staging();
    const auto d = st.carve(std::array<size_t, 2>{packed_bytes, out_bytes});
    st.upload(d[0], packed, packed_bytes);
    check_status(exl3cu_decode_inner(reinterpret_cast<const uint16_t *>(d[0]), k, n, first_column, column_count, bits,
                                     static_cast<unsigned>(codebook), reinterpret_cast<uint16_t *>(d[1]), st.stream));
    st.download(output, d[1], out_bytes);
    st.sync();
}

void hadamard128(float * values, size_t count) {
    if (count % 128) throw std::invalid_argument("H128 length must be a multiple of 128");
    if (!count) return;
    Staging & st = staging();
    const auto d = st.carve(std::array<size_t, 1>{count * 4});
    st.upload(d[0], values, count * 4);
    check_status(exl3cu_hadamard128(reinterpret_cast<float *>(d[0]), count, st.stream));
    st.download(values, d[0], count * 4);
    st.sync();
}

void reconstruct(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                 unsigned bits, Codebook codebook, uint16_t * output) {
    reconstruct_slice(packed, suh, svh, k, n, 0, n, bits, codebook, output);
}

void reconstruct_slice(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                       size_t first_column, size_t column_count, unsigned bits, Codebook codebook, uint16_t * output) {
    validate_shape(k, n, 128);
    if (first_column % 128 || column_count % 128)
        throw std::invalid_argument("H128 slices must align to 128 columns");
    validate(bits, codebook);
    if (!column_count || first_column > n || column_count > n - first_column)
        throw std::invalid_argument("Invalid EXL3 column slice");
    const size_t packed_bytes = k * n * bits / 8;
    const size_t out_bytes = k * column_count * 2;
    Staging & st = staging();
    const auto d = st.carve(std::array<size_t, 4>{packed_bytes, k * 2, n * 2, out_bytes});
    st.upload(d[0], packed, packed_bytes);
    st.upload(d[1], suh, k * 2);
    st.upload(d[2], svh, n * 2);
    check_status(exl3cu_reconstruct(reinterpret_cast<const uint16_t *>(d[0]), reinterpret_cast<const uint16_t *>(d[1]),
                                    reinterpret_cast<const uint16_t *>(d[2]), k, n, first_column, column_count, bits,
                                    static_cast<unsigned>(codebook), reinterpret_cast<uint16_t *>(d[3]), st.stream));
    st.download(output, d[3], out_bytes);
    st.sync();
}

}  // namespace exl3
