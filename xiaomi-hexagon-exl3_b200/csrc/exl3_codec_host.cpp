// exl3:: host API (include/exl3_codec.h) over the exl3cu C ABI.
//
// Same signatures, layouts and std::invalid_argument contract as the
// reference's src/exl3_codec.cpp; the work runs on the current CUDA device.
// Each call stages its host buffers in device memory, launches, and copies
// the result back on a private stream it synchronises before returning.
#include "exl3_codec.h"

#include <cuda_runtime.h>

#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>

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

// Device buffer owned for the duration of one call.
struct DeviceBuffer {
    void * p = nullptr;
    explicit DeviceBuffer(size_t bytes) { check_cuda(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc"); }
    ~DeviceBuffer() { cudaFree(p); }
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer & operator=(const DeviceBuffer &) = delete;
    template <class T> T * as() const { return static_cast<T *>(p); }
};

struct Stream {
    cudaStream_t s = nullptr;
    Stream() { check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate"); }
    ~Stream() { cudaStreamDestroy(s); }
    void sync() const { check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize"); }
};

void upload(void * dst, const void * src, size_t bytes, const Stream & st) {
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st.s), "copy to device");
}

void download(void * dst, const void * src, size_t bytes, const Stream & st) {
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st.s), "copy to host");
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
    Stream st;
    DeviceBuffer in(2), out(2);
    upload(in.p, &state, 2, st);
    check_status(exl3cu_decode_codebook(in.as<uint16_t>(), 1, static_cast<unsigned>(codebook), out.as<uint16_t>(),
                                        st.s));
    uint16_t r = 0;
    download(&r, out.p, 2, st);
    st.sync();
    return r;
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
    Stream st;
    DeviceBuffer dp(packed_bytes), dout(out_bytes);
    upload(dp.p, packed, packed_bytes, st);
    check_status(exl3cu_decode_inner(dp.as<uint16_t>(), k, n, first_column, column_count, bits,
                                     static_cast<unsigned>(codebook), dout.as<uint16_t>(), st.s));
    download(output, dout.p, out_bytes, st);
    st.sync();
}

void hadamard128(float * values, size_t count) {
    if (count % 128) throw std::invalid_argument("H128 length must be a multiple of 128");
    if (!count) return;
    Stream st;
    DeviceBuffer dv(count * 4);
    upload(dv.p, values, count * 4, st);
    check_status(exl3cu_hadamard128(dv.as<float>(), count, st.s));
    download(values, dv.p, count * 4, st);
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
    Stream st;
    DeviceBuffer dp(packed_bytes), dsu(k * 2), dsv(n * 2), dout(out_bytes);
    upload(dp.p, packed, packed_bytes, st);
    upload(dsu.p, suh, k * 2, st);
    upload(dsv.p, svh, n * 2, st);
    check_status(exl3cu_reconstruct(dp.as<uint16_t>(), dsu.as<uint16_t>(), dsv.as<uint16_t>(), k, n, first_column,
                                    column_count, bits, static_cast<unsigned>(codebook), dout.as<uint16_t>(), st.s));
    download(output, dout.p, out_bytes, st);
    st.sync();
}

}  // namespace exl3
