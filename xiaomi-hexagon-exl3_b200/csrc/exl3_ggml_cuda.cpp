// ggml_exl3_mul_mat and ggml_exl3_get_rows for ggml's CPU backend, executed
// on a B200 through the exl3cu C ABI.  Drop-in for the reference's
// src/exl3-ggml.cpp: same symbols, same tensor contracts, same GGML_ASSERT
// checks.
//  * mul_mat (src/exl3-ggml.cpp:51-92): src0 EXL3_4/6/8 [k, n] runtime
//    records, src1 F32/F16 [k, r1, r2, r3] with byte strides nb[], dst F32
//    [n, r1, r2, r3].
//  * get_rows (src/exl3-ggml.cpp:19-49): src0 as above, src1 I32 ids of any
//    shape (element r = row r / ne[0], column r % ne[0]), dst F32 with one
//    k-wide row per id (rows addressed through ne[1], ne[2] and nb[1..3]).
//
// ggml calls an op from nth threads with ith = 0..nth-1 and joins them on a
// barrier before the next op.  Thread 0 alone drives the GPU -- it uploads the
// weight on first sight, stages the activations, runs the operator and copies
// y back before returning (on the legacy default stream, synchronised); the
// other threads return at once and wait on ggml's barrier.
//
// Uploaded weights are cached by data pointer, type and shape plus a digest of
// the records (the first and last record in full and a strided sample of the
// rest), checked on every call: a model reloaded at the same address, or a
// second model reusing a freed buffer, gets its own upload and the stale one is
// freed.  ggml_exl3_release_weights() frees every cached upload (call it when a
// model is unloaded).
//
// Device: EXL3CU_DEVICE (default 0).  Built in a llama.cpp tree this file
// compiles against upstream's ggml.h / ggml-cpu-impl.h; the standalone build
// uses the stand-ins in csrc/ggml_stub.
#include "exl3-block.h"
#include "exl3cu.h"
#include "ggml-cpu-impl.h"
#include "ggml.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace {

struct Cached {
    exl3cu_weight * handle;
    uint64_t digest;
};
std::mutex g_mu;
std::map<std::tuple<const void *, int, int64_t, int64_t>, Cached> g_weights;

// A digest of the records, taken on every call: 8-byte words (the first and last 64 of the buffer
// and 64 sampled evenly across it) folded FNV-style, one multiply per word.  It changes when a
// different model occupies the same buffer (new weights differ in nearly every word) and costs well
// under a microsecond; hashing two whole records byte by byte had cost about 25 us per call.
uint64_t records_digest(const void * data, size_t bytes) {
    const unsigned char * p = static_cast<const unsigned char *>(data);
    const size_t words = bytes / 8;
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](size_t word) {
        uint64_t v;
        std::memcpy(&v, p + word * 8, 8);
        h = (h ^ v) * 1099511628211ull;
    };
    const size_t edge = words < 64 ? words : 64;
    for (size_t i = 0; i < edge; ++i) mix(i);
    for (size_t i = 0; i < edge; ++i) mix(words - edge + i);
    for (size_t i = 0; i < 64 && words; ++i) mix(i * (words - 1) / 63);
    return h;
}

int target_device() {
    const char * env = std::getenv("EXL3CU_DEVICE");
    return env ? std::atoi(env) : 0;
}

[[noreturn]] void die(const char * what, int rc) {
    std::fprintf(stderr, "exl3cu: %s failed (%s): %s\n", what, exl3cu_status_string(rc), exl3cu_last_error());
    std::abort();
}

exl3cu_weight * weight_for(const ggml_tensor * w, unsigned bits, size_t k, size_t n) {
    const auto key = std::make_tuple(static_cast<const void *>(w->data), int(w->type), int64_t(k), int64_t(n));
    const size_t bytes = (k / 128) * (n / 128) * exl3_group_bytes(bits);
    const uint64_t digest = records_digest(w->data, bytes);
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_weights.find(key);
    if (it != g_weights.end()) {
        if (it->second.digest == digest) return it->second.handle;
        exl3cu_weight_free(it->second.handle);  // other records now live at this address
        g_weights.erase(it);
    }
    exl3cu_weight * h = nullptr;
    int rc = exl3cu_weight_from_records(w->data, bytes, k, n, bits, EXL3CU_CB_MUL1, 0, 0, target_device(), &h);
    if (rc) die("uploading EXL3 weight", rc);
    g_weights[key] = Cached{h, digest};
    return h;
}

// Byte offset of row `row` of t, rows counted across ne[1], ne[2], ne[3].
size_t row_offset(const ggml_tensor * t, size_t row) {
    const size_t i1 = row % size_t(t->ne[1]);
    row /= size_t(t->ne[1]);
    const size_t i2 = row % size_t(t->ne[2]);
    const size_t i3 = row / size_t(t->ne[2]);
    return i1 * t->nb[1] + i2 * t->nb[2] + i3 * t->nb[3];
}

}  // namespace

extern "C" void ggml_exl3_get_rows(const ggml_compute_params * params, ggml_tensor * dst) {
    const ggml_tensor * weight = dst->src[0];
    const ggml_tensor * ids = dst->src[1];
    const size_t k = size_t(weight->ne[0]), n = size_t(weight->ne[1]);
    const unsigned bits = exl3_type_bits(weight->type);
    GGML_ASSERT(bits && k && n && k % 128 == 0 && n % 128 == 0 && weight->ne[2] == 1 && weight->ne[3] == 1);
    GGML_ASSERT(ids->type == GGML_TYPE_I32 && dst->type == GGML_TYPE_F32);
    if (params->ith != 0) return;
    const size_t count = size_t(ggml_nelements(ids));
    if (!count) return;
    GGML_ASSERT(dst->nb[0] == 4 && size_t(dst->ne[0]) >= k);
    std::vector<int32_t> id(count);
    for (size_t r = 0; r < count; ++r) {
        const size_t row = r / size_t(ids->ne[0]), col = r % size_t(ids->ne[0]);
        std::memcpy(&id[r], static_cast<const char *>(ids->data) + row_offset(ids, row) + col * ids->nb[0], 4);
        GGML_ASSERT(id[r] >= 0 && size_t(id[r]) < n);
    }
    exl3cu_weight * h = weight_for(weight, bits, k, n);
    // Rows of dst that are evenly spaced (the usual contiguous [k, count]
    // result) are written in place; otherwise through a contiguous buffer.
    bool even = true;
    const size_t stride = count > 1 ? row_offset(dst, 1) : k * 4;
    for (size_t r = 0; r < count && even; ++r) even = row_offset(dst, r) == r * stride;
    even = even && stride % 4 == 0 && stride >= k * 4;
    // one call per kMaxIds ids (the library's per-call limit)
    constexpr size_t kMaxIds = 65535;
    if (even) {
        for (size_t r0 = 0; r0 < count; r0 += kMaxIds) {
            const size_t c = count - r0 < kMaxIds ? count - r0 : kMaxIds;
            const int rc = exl3cu_get_rows_host(h, id.data() + r0, c,
                                                reinterpret_cast<float *>(static_cast<char *>(dst->data) + r0 * stride),
                                                stride / 4, 1, nullptr);
            if (rc) die("ggml_exl3_get_rows", rc);
        }
        return;
    }
    std::vector<float> tmp(count * k);
    for (size_t r0 = 0; r0 < count; r0 += kMaxIds) {
        const size_t c = count - r0 < kMaxIds ? count - r0 : kMaxIds;
        const int rc = exl3cu_get_rows_host(h, id.data() + r0, c, tmp.data() + r0 * k, k, 1, nullptr);
        if (rc) die("ggml_exl3_get_rows", rc);
    }
    for (size_t r = 0; r < count; ++r)
        std::memcpy(static_cast<char *>(dst->data) + row_offset(dst, r), tmp.data() + r * k, k * 4);
}

extern "C" void ggml_exl3_mul_mat(const ggml_compute_params * params, ggml_tensor * dst) {
    const ggml_tensor * weight = dst->src[0];
    const ggml_tensor * input = dst->src[1];
    const size_t k = size_t(weight->ne[0]), n = size_t(weight->ne[1]);
    const unsigned bits = exl3_type_bits(weight->type);
    GGML_ASSERT(bits && k % 128 == 0 && n % 128 == 0 && weight->ne[2] == 1 && weight->ne[3] == 1);
    GGML_ASSERT(input->type == GGML_TYPE_F32 || input->type == GGML_TYPE_F16);
    if (params->ith != 0) return;
    const size_t es = input->type == GGML_TYPE_F32 ? 4 : 2;
    GGML_ASSERT(size_t(input->ne[0]) == k && input->nb[0] == es && dst->nb[0] == 4 && size_t(dst->ne[0]) == n);
    GGML_ASSERT(input->nb[1] % es == 0 && dst->nb[1] % 4 == 0);
    exl3cu_weight * h = weight_for(weight, bits, k, n);
    const int dtype = input->type == GGML_TYPE_F32 ? EXL3CU_F32 : EXL3CU_F16;
    for (int64_t i3 = 0; i3 < input->ne[3]; ++i3) {
        for (int64_t i2 = 0; i2 < input->ne[2]; ++i2) {
            const char * x = static_cast<const char *>(input->data) + i2 * input->nb[2] + i3 * input->nb[3];
            char * y = static_cast<char *>(dst->data) + i2 * dst->nb[2] + i3 * dst->nb[3];
            const int rc = exl3cu_mul_mat_host(h, x, dtype, size_t(input->ne[1]), input->nb[1] / es,
                                               reinterpret_cast<float *>(y), dst->nb[1] / 4, 1, nullptr);
            if (rc) die("ggml_exl3_mul_mat", rc);
        }
    }
}

extern "C" void ggml_exl3_release_weights(void) {
    std::lock_guard<std::mutex> g(g_mu);
    for (auto & e : g_weights) exl3cu_weight_free(e.second.handle);
    g_weights.clear();
}
