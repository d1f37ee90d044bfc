// exl3::Model -- the reference reader's class interface (its
// include/exl3_model.h: constructor from a deployment directory, tensor_count,
// payload_bytes, hidden_size, vocab_size, bits_per_weight, embedding), backed
// by the B200 loader: the directory is validated with the same rules and
// messages, then every EXL3 matrix is uploaded to the CUDA device current at
// construction.  embedding(token) returns the same fp16 bits as the
// reference's reconstruct_slice-based lookup, computed on the GPU.
// Constructor failures throw std::runtime_error; embedding() throws
// std::invalid_argument for a token outside the vocabulary.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

struct exl3cu_model;

namespace exl3 {

class Model {
public:
    explicit Model(const std::string & directory);
    ~Model();
    Model(const Model &) = delete;
    Model & operator=(const Model &) = delete;
    size_t tensor_count() const;
    size_t payload_bytes() const;
    size_t hidden_size() const;
    size_t vocab_size() const;
    double bits_per_weight() const;
    std::vector<uint16_t> embedding(uint32_t token) const;
    // Not in the reference: the loader handle (weights of every matrix, the
    // device tensor arena) for the exl3cu_model_* C functions.
    exl3cu_model * handle() const;

private:
    struct Impl;
    std::unique_ptr<Impl> impl;
};

}  // namespace exl3
