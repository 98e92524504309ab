// forge/mtp.hpp — the reference's multi-token-prediction heads
// (include/forge/mtp.hpp:23-76 there) running on the GPU.
//
// Each head is a SwiGLU block of three Q4 matrices (gate, up: ff x d; down:
// d x ff; per-row fp32 scales); heads are chained: head h reads the hidden
// left by head h-1.  init_weights draws uniform(-1,1)/sqrt(d) values from
// rand() and quantizes them like the reference; forward runs every product
// on the device in the reference's summation order.
#ifndef FORGE_B200_MTP_HPP
#define FORGE_B200_MTP_HPP

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

#include "types.hpp"

namespace forge {

struct MTPConfig {
    uint32_t n_mtp_heads = 4;
    uint32_t n_embd = 2048;
    uint32_t n_vocab = 32000;
    uint32_t mtp_ff_dim = 2048;
};

class FORGE_API MTPHeads {
public:
    explicit MTPHeads(const MTPConfig& cfg);
    ~MTPHeads();
    MTPHeads(const MTPHeads&) = delete;
    MTPHeads& operator=(const MTPHeads&) = delete;

    void init_weights();
    // Logits of every head for one hidden vector; embedding_table is the tied
    // fp32 table [n_vocab][n_embd] (smaller: placeholder logits, as the reference).
    std::vector<std::vector<float>> forward(const float* hidden, const std::vector<float>& embedding_table) const;
    // 1 + the number of heads h >= 1 whose argmax equals `token`, stopping at
    // the first mismatch.
    int speculative_accept(int32_t token, const std::vector<std::vector<float>>& mtp_logits) const;
    // First index of the maximum.
    static int32_t argmax(const float* logits, uint32_t n);
    // Bytes of the heads' packed weights and scales.
    size_t memory_usage() const;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    MTPConfig cfg_;
};

}  // namespace forge

#endif  // FORGE_B200_MTP_HPP
