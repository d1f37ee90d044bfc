// exl3::Model used the way the reference's reader test uses it
// (tests/test_model_reader.cpp:37-79 of the reference), against
// deployment directories the Python test writes:
//   model_reader_check <fixture dir> <code16> <rejected dir>...
// <code16>: fp16 bits of fp16(decode_codebook(0, mul1) * 128), the value the
// reference test expects at row0[0].  Prints PASS and exits 0, or names the
// failed check and exits 1.
#include "exl3_model.h"

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

static int fail(const char * what) {
    std::printf("FAIL: %s\n", what);
    return 1;
}

int main(int argc, char ** argv) {
    if (argc < 3) return fail("usage");
    const unsigned code16 = unsigned(std::strtoul(argv[2], nullptr, 0));
    try {
        exl3::Model model(argv[1]);
        if (model.tensor_count() != 4 || model.payload_bytes() != 8708) return fail("Model payload inventory");
        if (model.hidden_size() != 128 || model.vocab_size() != 128) return fail("geometry");
        const auto row0 = model.embedding(0), row1 = model.embedding(1);
        if (row0 != model.embedding(0)) return fail("Cache preserves embedding");
        if (row0.size() != 128 || row0[0] != code16) return fail("Tied head basis and scale");
        for (size_t i = 1; i < row0.size(); ++i)
            if ((row0[i] & 0x7fffu) != 0) return fail("H128 column reduction");
        for (auto v : row1)
            if ((v & 0x7fffu) != 0) return fail("H128 nonzero column isolation");
        bool rejected = false;
        try {
            model.embedding(128);
        } catch (const std::invalid_argument &) {
            rejected = true;
        }
        if (!rejected) return fail("Reject token outside vocabulary");
    } catch (const std::exception & e) {
        std::printf("FAIL: %s\n", e.what());
        return 1;
    }
    for (int i = 3; i < argc; ++i) {
        bool rejected = false;
        try {
            exl3::Model model(argv[i]);
        } catch (const std::runtime_error &) {
            rejected = true;
        }
        if (!rejected) return fail("Malformed model must be rejected");
    }
    std::printf("PASS\n");
    return 0;
}
