// squeeze.hpp — reader of the reference's .squeeze weight files
// (src/quant_format.cpp:231-420, include/forge/quant_format.hpp:29-48): a
// 256-byte header, an index of 32-byte block records, zstd-compressed blocks.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "forge/types.hpp"

namespace forge {
namespace squeeze {

struct Block {
    uint32_t layer, matrix, rows, cols, compressed, original;
    uint8_t qtype;
    uint64_t offset;
};

// One block decoded as the reference's WeightLoader::load_block_with_scales
// returns it: int8 values (the reference's decoders read the stream from its
// first byte), per-row scales and the global scale.
struct Matrix {
    std::vector<int8_t> data;
    std::vector<float> row_scales;
    float global_scale = 1.0f;
    uint32_t rows = 0, cols = 0;
};

class File {
public:
    bool open(const std::string& path, std::string* err);
    const ModelConfig& config() const { return cfg_; }
    const Block* find(uint32_t layer, uint32_t matrix) const;
    // False with *err set when the block is missing or does not decode.
    bool load(uint32_t layer, uint32_t matrix, Matrix* out, std::string* err) const;

private:
    ModelConfig cfg_;
    std::vector<Block> blocks_;
    std::vector<uint8_t> bytes_;
};

}  // namespace squeeze
}  // namespace forge
