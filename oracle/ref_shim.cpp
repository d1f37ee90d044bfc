// Test infrastructure (the checker, never the product): plain C entry points
// around the reference's OWN compiled sources, so Python tests and the
// benchmark's CPU arm can call them through ctypes.  oracle/Makefile compiles
// this file together with the reference's unmodified src/exl3_codec.cpp and
// src/exl3-ggml.cpp into oracle/_ref/libexl3ref.so.
//
// Functions:
//   ref_decode_codebook  -> exl3::decode_codebook      (src/exl3_codec.cpp:68-86)
//   ref_decode_tile      -> exl3::decode_tile          (src/exl3_codec.cpp:92-115)
//   ref_decode_inner     -> exl3::decode_inner[_slice] (src/exl3_codec.cpp:123-145)
//   ref_hadamard128      -> exl3::hadamard128          (src/exl3_codec.cpp:147-167)
//   ref_reconstruct      -> exl3::reconstruct[_slice]  (src/exl3_codec.cpp:169-204)
//   ref_half_to_float / ref_float_to_half              (src/exl3_codec.cpp:21-66)
//   ref_ggml_mul_mat     -> ggml_exl3_mul_mat on nth std::threads, ith/nth split
//                           exactly as ggml's CPU backend calls it
//                           (src/exl3-ggml.cpp:51-92; patches/llama-exl3.patch:44-51)
//   ref_ggml_get_rows    -> ggml_exl3_get_rows         (src/exl3-ggml.cpp:19-49)
//   ref_loop_mul_mat     -> for bitrates the ggml types do not cover (1,2,3,5,7):
//                           the loop of src/exl3-ggml.cpp:51-92 restated over the
//                           reference's own exl3::decode_inner and exl3::hadamard128.
// Every entry returns 0 on success and 1 when the reference threw
// std::invalid_argument (its error contract, src/exl3_codec.cpp:12-19).
#include "exl3-block.h"
#include "exl3_codec.h"
#include "ggml-cpu-impl.h"
#include "ggml.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

namespace {

template <class F>
int guarded(F && fn) {
    try {
        fn();
        return 0;
    } catch (const std::invalid_argument &) {
        return 1;
    }
}

ggml_type exl3_ggml_type(unsigned bits) {
    return bits == 4 ? GGML_TYPE_EXL3_4 : bits == 6 ? GGML_TYPE_EXL3_6 : GGML_TYPE_EXL3_8;
}

}  // namespace

extern "C" {

float ref_half_to_float(uint16_t h) { return exl3::half_to_float(h); }
uint16_t ref_float_to_half(float f) { return exl3::float_to_half(f); }

int ref_decode_codebook(const uint16_t * states, size_t count, unsigned codebook, uint16_t * out) {
    return guarded([&] {
        if (codebook > 2) throw std::invalid_argument("codebook");
        for (size_t i = 0; i < count; ++i)
            out[i] = exl3::decode_codebook(states[i], static_cast<exl3::Codebook>(codebook));
    });
}

int ref_decode_tile(const uint16_t * packed, unsigned bits, unsigned codebook, uint16_t * out) {
    return guarded([&] { exl3::decode_tile(packed, bits, static_cast<exl3::Codebook>(codebook), out); });
}

int ref_decode_inner(const uint16_t * packed, size_t k, size_t n, size_t first_column, size_t column_count,
                     unsigned bits, unsigned codebook, uint16_t * out) {
    return guarded([&] {
        exl3::decode_inner_slice(packed, k, n, first_column, column_count, bits,
                                 static_cast<exl3::Codebook>(codebook), out);
    });
}

int ref_hadamard128(float * values, size_t count) {
    return guarded([&] { exl3::hadamard128(values, count); });
}

int ref_reconstruct(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                    size_t first_column, size_t column_count, unsigned bits, unsigned codebook, uint16_t * out) {
    return guarded([&] {
        exl3::reconstruct_slice(packed, suh, svh, k, n, first_column, column_count, bits,
                                static_cast<exl3::Codebook>(codebook), out);
    });
}

// records: the runtime group records (n/128 * k/128 records of 2048*bits+512 bytes,
// record (nb,kb) at index nb*(k/128)+kb).  x: rows contiguous rows of k values
// (f32 when x_is_f16 == 0, else f16 bits).  y: rows x n f32.
int ref_ggml_mul_mat(const void * records, unsigned bits, size_t k, size_t n, const void * x, int x_is_f16,
                     size_t rows, float * y, int nth) {
    if (bits != 4 && bits != 6 && bits != 8) return 1;
    if (nth < 1) nth = 1;
    ggml_tensor w{}, in{}, out{};
    w.type = exl3_ggml_type(bits);
    w.ne[0] = int64_t(k); w.ne[1] = int64_t(n); w.ne[2] = 1; w.ne[3] = 1;
    w.data = const_cast<void *>(records);
    const size_t es = x_is_f16 ? 2 : 4;
    in.type = x_is_f16 ? GGML_TYPE_F16 : GGML_TYPE_F32;
    in.ne[0] = int64_t(k); in.ne[1] = int64_t(rows); in.ne[2] = 1; in.ne[3] = 1;
    in.nb[0] = es; in.nb[1] = es * k; in.nb[2] = es * k * rows; in.nb[3] = in.nb[2];
    in.data = const_cast<void *>(x);
    out.type = GGML_TYPE_F32;
    out.ne[0] = int64_t(n); out.ne[1] = int64_t(rows); out.ne[2] = 1; out.ne[3] = 1;
    out.nb[0] = 4; out.nb[1] = 4 * n; out.nb[2] = 4 * n * rows; out.nb[3] = out.nb[2];
    out.data = y;
    out.src[0] = &w;
    out.src[1] = &in;
    std::vector<std::thread> pool;
    for (int ith = 1; ith < nth; ++ith) {
        pool.emplace_back([&, ith] {
            ggml_compute_params p{ith, nth, 0, nullptr};
            ggml_exl3_mul_mat(&p, &out);
        });
    }
    ggml_compute_params p0{0, nth, 0, nullptr};
    ggml_exl3_mul_mat(&p0, &out);
    for (auto & t : pool) t.join();
    return 0;
}

// ids: count int32 token ids; out: count x k f32 (one original-basis column each).
int ref_ggml_get_rows(const void * records, unsigned bits, size_t k, size_t n, const int32_t * ids, size_t count,
                      float * out_rows, int nth) {
    if (bits != 4 && bits != 6 && bits != 8) return 1;
    if (nth < 1) nth = 1;
    ggml_tensor w{}, idt{}, out{};
    w.type = exl3_ggml_type(bits);
    w.ne[0] = int64_t(k); w.ne[1] = int64_t(n); w.ne[2] = 1; w.ne[3] = 1;
    w.data = const_cast<void *>(records);
    idt.type = GGML_TYPE_I32;
    idt.ne[0] = int64_t(count); idt.ne[1] = 1; idt.ne[2] = 1; idt.ne[3] = 1;
    idt.nb[0] = 4; idt.nb[1] = 4 * count; idt.nb[2] = idt.nb[1]; idt.nb[3] = idt.nb[1];
    idt.data = const_cast<int32_t *>(ids);
    out.type = GGML_TYPE_F32;
    out.ne[0] = int64_t(k); out.ne[1] = int64_t(count); out.ne[2] = 1; out.ne[3] = 1;
    out.nb[0] = 4; out.nb[1] = 4 * k; out.nb[2] = 4 * k * count; out.nb[3] = out.nb[2];
    out.data = out_rows;
    out.src[0] = &w;
    out.src[1] = &idt;
    std::vector<std::thread> pool;
    for (int ith = 1; ith < nth; ++ith) {
        pool.emplace_back([&, ith] {
            ggml_compute_params p{ith, nth, 0, nullptr};
            ggml_exl3_get_rows(&p, &out);
        });
    }
    ggml_compute_params p0{0, nth, 0, nullptr};
    ggml_exl3_get_rows(&p0, &out);
    for (auto & t : pool) t.join();
    return 0;
}

// Same record layout and output as ref_ggml_mul_mat, for any bitrate 1..8 and any
// codebook: the three phases of src/exl3-ggml.cpp:51-92 (input rotation, per-group
// decode + fp32 accumulate, output rotation and scale), threaded over output column
// blocks the way ith/nth splits them, decoding through the reference's own
// exl3::decode_inner and rotating through exl3::hadamard128.
int ref_loop_mul_mat(const void * records, unsigned bits, unsigned codebook, size_t k, size_t n, const void * x,
                     int x_is_f16, size_t rows, float * y, int nth) {
    return guarded([&] {
        if (bits < 1 || bits > 8 || codebook > 2 || !k || !n || k % 128 || n % 128)
            throw std::invalid_argument("shape");
        const size_t group_bytes = 2048u * bits + 512u;
        const auto * base = static_cast<const uint8_t *>(records);
        std::vector<float> xh(rows * k);
        for (size_t kb = 0; kb < k / 128; ++kb) {
            const auto * su = reinterpret_cast<const uint16_t *>(base + kb * group_bytes + 2048u * bits);
            for (size_t r = 0; r < rows; ++r) {
                for (size_t j = 0; j < 128; ++j) {
                    float v;
                    if (x_is_f16) v = exl3::half_to_float(static_cast<const uint16_t *>(x)[r * k + kb * 128 + j]);
                    else v = static_cast<const float *>(x)[r * k + kb * 128 + j];
                    xh[r * k + kb * 128 + j] = v * exl3::half_to_float(su[j]);
                }
                exl3::hadamard128(xh.data() + r * k + kb * 128, 128);
            }
        }
        if (nth < 1) nth = 1;
        auto worker = [&](int ith) {
            std::vector<float> result(rows * 128);
            std::vector<uint16_t> decoded(128 * 128);
            for (size_t nb = size_t(ith); nb < n / 128; nb += size_t(nth)) {
                std::fill(result.begin(), result.end(), 0.0f);
                for (size_t kb = 0; kb < k / 128; ++kb) {
                    const auto * group = base + (nb * (k / 128) + kb) * group_bytes;
                    exl3::decode_inner(reinterpret_cast<const uint16_t *>(group), 128, 128, bits,
                                       static_cast<exl3::Codebook>(codebook), decoded.data());
                    for (size_t i = 0; i < 128; ++i)
                        for (size_t j = 0; j < 128; ++j) {
                            const float w = exl3::half_to_float(decoded[i * 128 + j]);
                            for (size_t r = 0; r < rows; ++r) result[r * 128 + j] += xh[r * k + kb * 128 + i] * w;
                        }
                }
                const auto * sv = reinterpret_cast<const uint16_t *>(base + nb * (k / 128) * group_bytes + 2048u * bits + 256u);
                for (size_t r = 0; r < rows; ++r) {
                    exl3::hadamard128(result.data() + r * 128, 128);
                    for (size_t j = 0; j < 128; ++j) y[r * n + nb * 128 + j] = result[r * 128 + j] * exl3::half_to_float(sv[j]);
                }
            }
        };
        std::vector<std::thread> pool;
        for (int ith = 1; ith < nth; ++ith) pool.emplace_back(worker, ith);
        worker(0);
        for (auto & t : pool) t.join();
    });
}

}  // extern "C"
