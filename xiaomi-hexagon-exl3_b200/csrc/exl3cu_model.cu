// Model loader: a deployment directory (model.safetensors + hexagon-exl3.json)
// into persistent device buffers on one GPU.
//
// Validation follows exl3::Model (src/exl3_model.cpp:79-157) rule for rule and
// in the same order, with the same messages:
//  * safetensors header: 8-byte little-endian length <= 64 MiB and inside the
//    file (:81-83); dtypes F16/BF16/I16/F32/I32 (:87-92); dimensions positive
//    integers, element count without overflow (:93-98); a [begin, end) pair of
//    non-negative integers whose length is elements x width and which lies in
//    the payload (:99-103); spans that tile the payload from 0 with no gap or
//    overlap (:109-114).
//  * manifest: format "hexagon-exl3", version 1, kv_cache "f16" (:115-119); a
//    tied_linear / original / token_axis 1 input embedding (:120-123); hidden
//    and vocab sizes multiples of 128 up to 16384 / 1048576 (:124-126);
//    weight_payload_bytes equal to the payload and payload x 8 /
//    reference_parameter_count <= 5.0 bits per weight (:127-130).
//  * the head named by input_embedding.source: I16 trellis [k/16, n/16,
//    16 x bits] with bits 1..8, F16 suh [k] and svh [n] (:131-139); codebook
//    markers .mul1 = 0x83dcd12d or .mcg = 0xcbac1fed as 4-byte I32, never both;
//    neither means 3inst (:140-156).
// Stricter than the reference: a key repeated in a JSON object and a "shape"
// that is not an array are rejected (nlohmann/json would keep the last
// duplicate and iterate a scalar as one dimension).
//
// Beyond the reference's reader, which keeps only the head: every tensor
// X.trellis (except the exllamav3 embedding form that has an X.signs
// companion, tools/inspect_model.py:73-85) is an EXL3 matrix, checked as
// tools/inspect_model.py:86-94 does (3-D I16, last dimension 16 x bits, bits
// 1..8) plus what the device operator needs (in and out features multiples of
// 128, F16 X.suh [k] and X.svh [n], the head's marker rules).  Each matrix is
// uploaded at its own bit width into a persistent weight handle (LSC layout,
// one copy of suh and svh -- the runtime records' duplicated scales are not
// reproduced).  Every other tensor is copied as-is into one device arena,
// each at a 256-byte aligned offset.
#include "exl3_model.h"
#include "exl3cu.h"
#include "exl3cu_internal.h"
#include "exl3cu_json.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <fstream>
#include <limits>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

using namespace exl3cu;

namespace {

struct LoadError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Read-only private mapping of a file (src/exl3_model.cpp:22-43).
struct Mapping {
    int fd = -1;
    size_t size = 0;
    const uint8_t * data = nullptr;
    explicit Mapping(const std::string & path) {
        fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) throw LoadError("Cannot open model weights");
        struct stat st{};
        if (fstat(fd, &st) || st.st_size < 8) {
            close(fd);
            fd = -1;
            throw LoadError("Invalid weight file size");
        }
        size = size_t(st.st_size);
        void * p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            close(fd);
            fd = -1;
            throw LoadError("Cannot map model weights");
        }
        data = static_cast<const uint8_t *>(p);
    }
    ~Mapping() {
        if (data) munmap(const_cast<uint8_t *>(data), size);
        if (fd >= 0) close(fd);
    }
    Mapping(const Mapping &) = delete;
    Mapping & operator=(const Mapping &) = delete;
};

// src/exl3_model.cpp:45-50: a non-negative integer, zero only where allowed.
size_t positive_integer(const json::Value & v, bool zero_allowed = false) {
    if (!v.is_int()) throw LoadError("Expected an integer dimension or offset");
    if (v.i < 0 || (v.i == 0 && !zero_allowed)) throw LoadError("Invalid dimension or offset");
    return size_t(v.i);
}

int dtype_code(const std::string & s, size_t * width) {
    if (s == "F16") { *width = 2; return EXL3CU_ST_F16; }
    if (s == "BF16") { *width = 2; return EXL3CU_ST_BF16; }
    if (s == "I16") { *width = 2; return EXL3CU_ST_I16; }
    if (s == "F32") { *width = 4; return EXL3CU_ST_F32; }
    if (s == "I32") { *width = 4; return EXL3CU_ST_I32; }
    return -1;
}

constexpr uint32_t kMul1Marker = 0x83dcd12du;
constexpr uint32_t kMcgMarker = 0xcbac1fedu;

}  // namespace

struct exl3cu_model {
    struct Tensor {
        std::string name;
        int dtype;
        std::vector<size_t> shape;
        size_t begin, end;               // byte offsets in the payload
        long matrix = -1;                // index of the EXL3 matrix this tensor belongs to
        size_t arena_offset = SIZE_MAX;  // plain tensors: offset in the device arena
    };
    struct Matrix {
        std::string name;  // prefix of X.trellis
        size_t k, n;
        unsigned bits, codebook;
        size_t trellis, suh, svh;  // tensor indices
        exl3cu_weight * w = nullptr;
    };

    int device = -1;
    bool uploaded = false;
    size_t payload = 0, parameters = 0, hidden = 0, vocab = 0, head = 0;
    std::vector<Tensor> tensors;  // sorted by name
    std::unordered_map<std::string, size_t> tensor_index;
    std::vector<Matrix> matrices;  // sorted by name
    std::unordered_map<std::string, size_t> matrix_index;
    void * arena = nullptr;
    size_t arena_bytes = 0;
    int32_t * d_token = nullptr;  // embedding() scratch: one id and k fp16 values
    uint16_t * d_embed = nullptr;
    std::mutex embed_mu;

    const Tensor & tensor(const std::string & key) const {
        auto it = tensor_index.find(key);
        if (it == tensor_index.end()) throw LoadError("Missing model tensor: " + key);
        return tensors[it->second];
    }
    const Tensor * find(const std::string & key) const {
        auto it = tensor_index.find(key);
        return it == tensor_index.end() ? nullptr : &tensors[it->second];
    }

    void release() {
        int prev = -1;
        const bool switched = device >= 0 && cudaGetDevice(&prev) == cudaSuccess && prev != device &&
                              cudaSetDevice(device) == cudaSuccess;
        for (auto & m : matrices) {
            if (m.w) weight_free_owned(m.w);
            m.w = nullptr;
        }
        if (arena) cudaFree(arena);
        if (d_token) cudaFree(d_token);
        if (d_embed) cudaFree(d_embed);
        arena = nullptr;
        d_token = nullptr;
        d_embed = nullptr;
        if (switched) cudaSetDevice(prev);
    }
    ~exl3cu_model() { release(); }
};

namespace {

// Codebook of the matrix with prefix `prefix` from its marker tensors
// (src/exl3_model.cpp:140-156).
unsigned read_codebook(const exl3cu_model & m, const Mapping & map, size_t data_begin, const std::string & prefix,
                       const char * what) {
    const auto * mul1 = m.find(prefix + ".mul1");
    const auto * mcg = m.find(prefix + ".mcg");
    if (mul1 && mcg) throw LoadError(std::string("Ambiguous ") + what + " codebook");
    const auto * marker = mul1 ? mul1 : mcg;
    if (!marker) return EXL3CU_CB_3INST;
    if (marker->dtype != EXL3CU_ST_I32 || marker->end - marker->begin != 4) throw LoadError("Invalid codebook marker");
    uint32_t value;
    std::memcpy(&value, map.data + data_begin + marker->begin, 4);
    if (mul1) {
        if (value != kMul1Marker) throw LoadError("Unsupported mul1 codebook multiplier");
        return EXL3CU_CB_MUL1;
    }
    if (value != kMcgMarker) throw LoadError("Unsupported mcg codebook multiplier");
    return EXL3CU_CB_MCG;
}

std::string read_text(const std::string & path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw LoadError("Cannot open deployment manifest");
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// Header, spans, manifest, head and matrices; no device work.
void validate(exl3cu_model & m, const Mapping & map, const std::string & directory, size_t * data_begin_out) {
    uint64_t header_size = 0;
    for (unsigned i = 0; i < 8; ++i) header_size |= uint64_t(map.data[i]) << (i * 8);
    if (header_size > 64u * 1024 * 1024 || header_size > map.size - 8) throw LoadError("Invalid safetensors header length");
    const char * hb = reinterpret_cast<const char *>(map.data + 8);
    const json::Value header = json::parse(hb, hb + header_size);
    if (!header.is_object()) throw LoadError("Invalid safetensors header");
    const size_t data_begin = 8 + size_t(header_size);
    const size_t payload_size = map.size - data_begin;
    std::vector<std::pair<size_t, size_t>> spans;
    for (const auto & member : header.members) {
        if (member.first == "__metadata__") continue;
        const json::Value & info = member.second;
        exl3cu_model::Tensor t;
        t.name = member.first;
        const json::Value & dt = info.at("dtype");
        if (!dt.is_string()) throw LoadError("Unsupported model dtype");
        size_t width = 0;
        t.dtype = dtype_code(dt.s, &width);
        if (t.dtype < 0) throw LoadError("Unsupported model dtype");
        const json::Value & shape = info.at("shape");
        if (!shape.is_array()) throw LoadError("Expected an integer dimension or offset");
        size_t elements = 1;
        for (const auto & d : shape.items) {
            const size_t dim = positive_integer(d);
            if (elements > std::numeric_limits<size_t>::max() / dim) throw LoadError("Tensor shape overflow");
            elements *= dim;
            t.shape.push_back(dim);
        }
        const json::Value & offsets = info.at("data_offsets");
        if (!offsets.is_array() || offsets.items.size() != 2) throw LoadError("Invalid tensor offset pair");
        const size_t begin = positive_integer(offsets.items[0], true), end = positive_integer(offsets.items[1], true);
        if (end < begin || end > payload_size || elements > std::numeric_limits<size_t>::max() / width ||
            end - begin != elements * width)
            throw LoadError("Invalid tensor data span");
        t.begin = begin;
        t.end = end;
        spans.emplace_back(begin, end);
        m.tensors.push_back(std::move(t));
    }
    std::sort(spans.begin(), spans.end());
    for (const auto & s : spans) {
        if (s.first != m.payload) throw LoadError("Overlapping or missing tensor data");
        m.payload = s.second;
    }
    if (m.payload != payload_size) throw LoadError("Unaccounted model payload");
    std::sort(m.tensors.begin(), m.tensors.end(),
              [](const exl3cu_model::Tensor & a, const exl3cu_model::Tensor & b) { return a.name < b.name; });
    for (size_t i = 0; i < m.tensors.size(); ++i) m.tensor_index.emplace(m.tensors[i].name, i);

    const std::string text = read_text(directory + "/hexagon-exl3.json");
    const json::Value manifest = json::parse(text);
    if (!manifest.is_object()) throw LoadError("Unsupported deployment manifest");
    if (!manifest.at("format").equals_string("hexagon-exl3") || !manifest.at("version").equals_int(1) ||
        !manifest.at("kv_cache").equals_string("f16"))
        throw LoadError("Unsupported deployment manifest");
    const json::Value & emb = manifest.at("input_embedding");
    if (!emb.at("type").equals_string("tied_linear") || !emb.at("basis").equals_string("original") ||
        !emb.at("token_axis").equals_int(1))
        throw LoadError("Unsupported embedding alias");
    const size_t k = positive_integer(emb.at("hidden_size"));
    const size_t n = positive_integer(emb.at("vocab_size"));
    if (k % 128 || n % 128 || k > 16384 || n > 1048576) throw LoadError("Invalid embedding geometry");
    m.hidden = k;
    m.vocab = n;
    m.parameters = positive_integer(manifest.at("reference_parameter_count"));
    if (positive_integer(manifest.at("weight_payload_bytes")) != m.payload ||
        double(m.payload) * 8 / double(m.parameters) > 5.0)
        throw LoadError("Model payload or budget mismatch");
    const json::Value & source = emb.at("source");
    if (!source.is_string()) throw LoadError("Unsupported embedding alias");
    const std::string head = source.s;
    const auto & packed = m.tensor(head + ".trellis");
    if (packed.dtype != EXL3CU_ST_I16 || packed.shape.size() != 3 || packed.shape[0] != k / 16 ||
        packed.shape[1] != n / 16 || packed.shape[2] % 16 || packed.shape[2] < 16 || packed.shape[2] > 128)
        throw LoadError("Invalid head trellis");
    for (const auto & e : {std::make_pair(std::string("suh"), k), std::make_pair(std::string("svh"), n)}) {
        const auto & sc = m.tensor(head + "." + e.first);
        if (sc.dtype != EXL3CU_ST_F16 || sc.shape != std::vector<size_t>{e.second}) throw LoadError("Invalid head scale");
    }
    read_codebook(m, map, data_begin, head, "head");

    // Every EXL3 matrix (the head included).
    const std::string suffix = ".trellis";
    for (size_t i = 0; i < m.tensors.size(); ++i) {
        const auto & t = m.tensors[i];
        if (t.name.size() <= suffix.size() || t.name.compare(t.name.size() - suffix.size(), suffix.size(), suffix))
            continue;
        const std::string prefix = t.name.substr(0, t.name.size() - suffix.size());
        if (m.find(prefix + ".signs")) continue;  // exllamav3 embedding form: kept as plain tensors
        if (t.dtype != EXL3CU_ST_I16 || t.shape.size() != 3 || t.shape[2] % 16)
            throw LoadError("Unsupported EXL3 trellis: " + t.name);
        const size_t bits = t.shape[2] / 16;
        if (bits < 1 || bits > 8) throw LoadError("Invalid EXL3 bitrate: " + t.name);
        exl3cu_model::Matrix mx;
        mx.name = prefix;
        mx.k = t.shape[0] * 16;
        mx.n = t.shape[1] * 16;
        mx.bits = unsigned(bits);
        if (mx.k % 128 || mx.n % 128)
            throw LoadError("EXL3 matrix " + prefix + ": in and out features must be multiples of 128");
        const auto * su = m.find(prefix + ".suh");
        const auto * sv = m.find(prefix + ".svh");
        if (!su || !sv || su->dtype != EXL3CU_ST_F16 || sv->dtype != EXL3CU_ST_F16 ||
            su->shape != std::vector<size_t>{mx.k} || sv->shape != std::vector<size_t>{mx.n})
            throw LoadError("Invalid EXL3 scales: " + prefix);
        mx.codebook = read_codebook(m, map, data_begin, prefix, "matrix");
        mx.trellis = i;
        mx.suh = m.tensor_index.at(prefix + ".suh");
        mx.svh = m.tensor_index.at(prefix + ".svh");
        m.matrices.push_back(std::move(mx));
    }
    std::sort(m.matrices.begin(), m.matrices.end(),
              [](const exl3cu_model::Matrix & a, const exl3cu_model::Matrix & b) { return a.name < b.name; });
    for (size_t j = 0; j < m.matrices.size(); ++j) {
        const auto & mx = m.matrices[j];
        m.matrix_index.emplace(mx.name, j);
        const long idx = long(j);
        m.tensors[mx.trellis].matrix = idx;
        m.tensors[mx.suh].matrix = idx;
        m.tensors[mx.svh].matrix = idx;
        for (const char * mk : {".mul1", ".mcg"}) {
            auto it = m.tensor_index.find(mx.name + mk);
            if (it != m.tensor_index.end()) m.tensors[it->second].matrix = idx;
        }
    }
    m.head = m.matrix_index.at(head);
    *data_begin_out = data_begin;
}

// Plain tensors into the arena, matrices into weight handles.
int upload(exl3cu_model & m, const Mapping & map, size_t data_begin) {
    size_t off = 0;
    for (auto & t : m.tensors) {
        if (t.matrix >= 0) continue;
        t.arena_offset = off;
        off += (t.end - t.begin + 255) & ~size_t(255);
    }
    m.arena_bytes = off;
    cudaError_t e = cudaSuccess;
    if (off) e = cudaMalloc(&m.arena, off);
    if (e == cudaSuccess) e = cudaMalloc(&m.d_token, 256);
    if (e == cudaSuccess) e = cudaMalloc(&m.d_embed, m.hidden * sizeof(uint16_t));
    if (e != cudaSuccess) return api_cuda_fail(e, "allocating model buffers");
    for (const auto & t : m.tensors) {
        if (t.matrix >= 0) continue;
        e = cudaMemcpy(static_cast<char *>(m.arena) + t.arena_offset, map.data + data_begin + t.begin, t.end - t.begin,
                       cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return api_cuda_fail(e, "copying model tensors");
    }
    for (auto & mx : m.matrices) {
        const auto * tr = reinterpret_cast<const uint16_t *>(map.data + data_begin + m.tensors[mx.trellis].begin);
        const auto * su = reinterpret_cast<const uint16_t *>(map.data + data_begin + m.tensors[mx.suh].begin);
        const auto * sv = reinterpret_cast<const uint16_t *>(map.data + data_begin + m.tensors[mx.svh].begin);
        exl3cu_weight * w = nullptr;
        const int rc = exl3cu_weight_from_trellis(tr, su, sv, mx.k, mx.n, mx.bits, mx.codebook, 0, 0, m.device, &w);
        if (rc) {
            const std::string why = exl3cu_last_error();
            return api_fail(rc, ("uploading EXL3 matrix " + mx.name + ": " + why).c_str());
        }
        weight_set_model_owned(w);
        mx.w = w;
    }
    m.uploaded = true;
    return EXL3CU_OK;
}

}  // namespace

extern "C" {

int exl3cu_model_open(const char * directory, int device, unsigned flags, exl3cu_model ** out) {
    if (!directory || !out) return api_fail(EXL3CU_INVALID_ARGUMENT, "directory and out are required");
    *out = nullptr;
    if (flags & ~unsigned(EXL3CU_MODEL_VALIDATE_ONLY)) return api_fail(EXL3CU_INVALID_ARGUMENT, "unknown flags");
    const bool validate_only = flags & EXL3CU_MODEL_VALIDATE_ONLY;
    auto * m = new (std::nothrow) exl3cu_model();
    if (!m) return api_fail(EXL3CU_OUT_OF_MEMORY, "host allocation");
    try {
        const std::string dir(directory);
        Mapping map(dir + "/model.safetensors");
        size_t data_begin = 0;
        validate(*m, map, dir, &data_begin);
        if (!validate_only) {
            int ndev = 0;
            if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
                (void)cudaGetLastError();
                delete m;
                return api_fail(EXL3CU_INVALID_ARGUMENT, ("cannot select device " + std::to_string(device)).c_str());
            }
            m->device = device;
            int prev = -1;
            cudaGetDevice(&prev);
            if (prev != device) cudaSetDevice(device);
            const int rc = upload(*m, map, data_begin);
            if (prev >= 0 && prev != device) cudaSetDevice(prev);
            if (rc) {
                delete m;
                return rc;
            }
        }
    } catch (const std::exception & e) {
        delete m;
        return api_fail(EXL3CU_INVALID_ARGUMENT, e.what());
    }
    *out = m;
    return EXL3CU_OK;
}

int exl3cu_model_free(exl3cu_model * m) {
    delete m;
    return EXL3CU_OK;
}

int exl3cu_model_info(const exl3cu_model * m, size_t * tensor_count, size_t * payload_bytes, size_t * hidden_size,
                      size_t * vocab_size, size_t * parameter_count, double * bits_per_weight) {
    if (!m) return api_fail(EXL3CU_INVALID_ARGUMENT, "model handle is NULL");
    if (tensor_count) *tensor_count = m->tensors.size();
    if (payload_bytes) *payload_bytes = m->payload;
    if (hidden_size) *hidden_size = m->hidden;
    if (vocab_size) *vocab_size = m->vocab;
    if (parameter_count) *parameter_count = m->parameters;
    if (bits_per_weight) *bits_per_weight = double(m->payload) * 8 / double(m->parameters);
    return EXL3CU_OK;
}

size_t exl3cu_model_matrix_count(const exl3cu_model * m) { return m ? m->matrices.size() : 0; }

int exl3cu_model_matrix(const exl3cu_model * m, size_t index, const char ** name, size_t * k, size_t * n,
                        unsigned * bits, unsigned * codebook, exl3cu_weight ** weight) {
    if (!m) return api_fail(EXL3CU_INVALID_ARGUMENT, "model handle is NULL");
    if (index >= m->matrices.size()) return api_fail(EXL3CU_INVALID_ARGUMENT, "matrix index out of range");
    const auto & mx = m->matrices[index];
    if (name) *name = mx.name.c_str();
    if (k) *k = mx.k;
    if (n) *n = mx.n;
    if (bits) *bits = mx.bits;
    if (codebook) *codebook = mx.codebook;
    if (weight) *weight = mx.w;
    return EXL3CU_OK;
}

int exl3cu_model_find_matrix(const exl3cu_model * m, const char * name, size_t * index) {
    if (!m || !name || !index) return api_fail(EXL3CU_INVALID_ARGUMENT, "model, name and index are required");
    auto it = m->matrix_index.find(name);
    if (it == m->matrix_index.end())
        return api_fail(EXL3CU_INVALID_ARGUMENT, (std::string("no EXL3 matrix named ") + name).c_str());
    *index = it->second;
    return EXL3CU_OK;
}

int exl3cu_model_head(const exl3cu_model * m, size_t * index) {
    if (!m || !index) return api_fail(EXL3CU_INVALID_ARGUMENT, "model and index are required");
    *index = m->head;
    return EXL3CU_OK;
}

int exl3cu_model_tensor(const exl3cu_model * m, size_t index, const char ** name, int * dtype, size_t * ndim,
                        const size_t ** shape, size_t * bytes, void ** d_data) {
    if (!m) return api_fail(EXL3CU_INVALID_ARGUMENT, "model handle is NULL");
    if (index >= m->tensors.size()) return api_fail(EXL3CU_INVALID_ARGUMENT, "tensor index out of range");
    const auto & t = m->tensors[index];
    if (name) *name = t.name.c_str();
    if (dtype) *dtype = t.dtype;
    if (ndim) *ndim = t.shape.size();
    if (shape) *shape = t.shape.data();
    if (bytes) *bytes = t.end - t.begin;
    if (d_data)
        *d_data = (m->uploaded && t.matrix < 0) ? static_cast<char *>(m->arena) + t.arena_offset : nullptr;
    return EXL3CU_OK;
}

int exl3cu_model_find_tensor(const exl3cu_model * m, const char * name, size_t * index) {
    if (!m || !name || !index) return api_fail(EXL3CU_INVALID_ARGUMENT, "model, name and index are required");
    auto it = m->tensor_index.find(name);
    if (it == m->tensor_index.end())
        return api_fail(EXL3CU_INVALID_ARGUMENT, (std::string("Missing model tensor: ") + name).c_str());
    *index = it->second;
    return EXL3CU_OK;
}

int exl3cu_model_embedding(exl3cu_model * m, uint32_t token, uint16_t * h_out) {
    if (!m || !h_out) return api_fail(EXL3CU_INVALID_ARGUMENT, "model and out are required");
    if (token >= m->vocab) return api_fail(EXL3CU_INVALID_ARGUMENT, "Token ID outside vocabulary");
    if (!m->uploaded) return api_fail(EXL3CU_NO_SUPPORT, "model was opened for validation only");
    std::lock_guard<std::mutex> lock(m->embed_mu);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != m->device) cudaSetDevice(m->device);
    const WeightGeometry g = weight_geometry(m->matrices[m->head].w);
    const int32_t id = int32_t(token);
    cudaError_t e = cudaMemcpy(m->d_token, &id, sizeof(id), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = launch_get_rows(g.lsc, g.su, g.sv, g.k, g.n_local, g.bits, g.codebook, m->d_token, 1, m->d_embed, g.k, true,
                            nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(h_out, m->d_embed, g.k * sizeof(uint16_t), cudaMemcpyDeviceToHost);
    if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return api_cuda_fail(e, "embedding lookup");
    return EXL3CU_OK;
}

int exl3cu_model_embed(const exl3cu_model * m, const int32_t * d_ids, size_t count, float * d_out,
                       size_t out_row_stride, void * stream) {
    if (!m) return api_fail(EXL3CU_INVALID_ARGUMENT, "model handle is NULL");
    if (!m->uploaded) return api_fail(EXL3CU_NO_SUPPORT, "model was opened for validation only");
    return exl3cu_get_rows(m->matrices[m->head].w, d_ids, count, d_out, out_row_stride, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// exl3::Model (include/exl3_model.h): the reference class's interface over the
// handle above, on the CUDA device current at construction.

namespace exl3 {

struct Model::Impl {
    exl3cu_model * h = nullptr;
    ~Impl() { exl3cu_model_free(h); }
};

Model::Model(const std::string & directory) : impl(std::make_unique<Impl>()) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        (void)cudaGetLastError();
        device = 0;
    }
    if (exl3cu_model_open(directory.c_str(), device, 0, &impl->h)) throw std::runtime_error(exl3cu_last_error());
}

Model::~Model() = default;

size_t Model::tensor_count() const { return impl->h->tensors.size(); }
size_t Model::payload_bytes() const { return impl->h->payload; }
size_t Model::hidden_size() const { return impl->h->hidden; }
size_t Model::vocab_size() const { return impl->h->vocab; }
double Model::bits_per_weight() const { return double(impl->h->payload) * 8 / double(impl->h->parameters); }

std::vector<uint16_t> Model::embedding(uint32_t token) const {
    if (token >= impl->h->vocab) throw std::invalid_argument("Token ID outside vocabulary");
    std::vector<uint16_t> out(impl->h->hidden);
    if (exl3cu_model_embedding(impl->h, token, out.data())) throw std::runtime_error(exl3cu_last_error());
    return out;
}

exl3cu_model * Model::handle() const { return impl->h; }

}  // namespace exl3
