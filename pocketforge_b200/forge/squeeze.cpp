// squeeze.cpp — .squeeze reader.  Decompression uses the system's libzstd
// (loaded at run time); the nibble / crumb decoding runs on the GPU through
// the forge:: dequant functions, exactly as the reference's loader decodes.
#include "squeeze.hpp"

#include <dlfcn.h>

#include <cstring>
#include <fstream>

#include "forge/matmul_neon.hpp"

namespace forge {
namespace squeeze {

namespace {

struct Zstd {
    size_t (*decompress)(void*, size_t, const void*, size_t) = nullptr;
    unsigned (*is_error)(size_t) = nullptr;
    bool ok = false;
};

const Zstd& zstd() {
    static Zstd z = [] {
        Zstd r;
        void* h = dlopen("libzstd.so.1", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libzstd.so", RTLD_NOW | RTLD_LOCAL);
        if (h) {
            r.decompress = reinterpret_cast<size_t (*)(void*, size_t, const void*, size_t)>(dlsym(h, "ZSTD_decompress"));
            r.is_error = reinterpret_cast<unsigned (*)(size_t)>(dlsym(h, "ZSTD_isError"));
            r.ok = r.decompress && r.is_error;
        }
        return r;
    }();
    return z;
}

template <class T>
T rd(const uint8_t* p) {
    T v;
    std::memcpy(&v, p, sizeof(T));
    return v;
}

}  // namespace

bool File::open(const std::string& path, std::string* err) {
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        *err = "cannot open " + path;
        return false;
    }
    bytes_.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
    // Header (256 bytes, packed): magic[8] "FORGE", version, n_blocks, the
    // config (n_layers, n_embd, n_heads, n_kv_heads, n_ff, n_vocab,
    // max_seq_len, mtp_heads), index offset and size (u64).
    if (bytes_.size() < 256 || std::memcmp(bytes_.data(), "FORGE", 5) != 0) {
        *err = path + " is not a .squeeze file";
        return false;
    }
    const uint8_t* h = bytes_.data();
    const uint32_t n_blocks = rd<uint32_t>(h + 12);
    cfg_.n_layers = rd<uint32_t>(h + 16);
    cfg_.n_embd = rd<uint32_t>(h + 20);
    cfg_.n_heads = rd<uint32_t>(h + 24);
    cfg_.n_kv_heads = rd<uint32_t>(h + 28);
    cfg_.n_ff = rd<uint32_t>(h + 32);
    cfg_.n_vocab = rd<uint32_t>(h + 36);
    cfg_.max_seq_len = rd<uint32_t>(h + 40);
    cfg_.mtp_heads = rd<uint32_t>(h + 44);
    const uint64_t index = rd<uint64_t>(h + 48);
    // Index records (32 bytes, natural alignment): layer, matrix, rows, cols,
    // compressed size, original size, quant type (u8 + 3 padding), offset.
    if (index + (uint64_t)n_blocks * 32 > bytes_.size()) {
        *err = path + ": index beyond the end of the file";
        return false;
    }
    blocks_.resize(n_blocks);
    for (uint32_t i = 0; i < n_blocks; i++) {
        const uint8_t* r = bytes_.data() + index + (size_t)i * 32;
        Block& b = blocks_[i];
        b.layer = rd<uint32_t>(r);
        b.matrix = rd<uint32_t>(r + 4);
        b.rows = rd<uint32_t>(r + 8);
        b.cols = rd<uint32_t>(r + 12);
        b.compressed = rd<uint32_t>(r + 16);
        b.original = rd<uint32_t>(r + 20);
        b.qtype = r[24];
        b.offset = rd<uint32_t>(r + 28);
        if (b.offset + (uint64_t)b.compressed > bytes_.size()) {
            *err = path + ": block data beyond the end of the file";
            return false;
        }
    }
    return true;
}

const Block* File::find(uint32_t layer, uint32_t matrix) const {
    for (const Block& b : blocks_)
        if (b.layer == layer && b.matrix == matrix) return &b;  // the first match, as the reference
    return nullptr;
}

bool File::load(uint32_t layer, uint32_t matrix, Matrix* out, std::string* err) const {
    const Block* b = find(layer, matrix);
    if (!b) {
        *err = "no block (layer " + std::to_string(layer) + ", matrix " + std::to_string(matrix) + ")";
        return false;
    }
    const Zstd& z = zstd();
    if (!z.ok) {
        *err = "libzstd.so.1 not found";
        return false;
    }
    std::vector<uint8_t> raw(b->original);
    const size_t got = z.decompress(raw.data(), raw.size(), bytes_.data() + b->offset, b->compressed);
    if (z.is_error(got)) {
        *err = "zstd could not decompress block (" + std::to_string(layer) + ", " + std::to_string(matrix) + ")";
        return false;
    }
    const uint32_t n = b->rows * b->cols;
    out->rows = b->rows;
    out->cols = b->cols;
    out->data.assign(n, 0);
    out->global_scale = 1.0f;
    switch (b->qtype) {
        case 0: {  // Q8: per 32 values a float scale then 32 int8 (src/quant_format.cpp:361-388)
            const uint32_t nb = (n + 31) / 32, bpr = (b->cols + 31) / 32;
            out->row_scales.assign(b->rows, 0.0f);
            const uint8_t* p = raw.data();
            for (uint32_t k = 0; k < nb; k++) {
                if ((size_t)(p - raw.data()) + 36 > raw.size()) break;
                const float s = rd<float>(p);
                p += 4;
                if (bpr) out->row_scales[k / bpr] += s;
                const uint32_t s0 = k * 32, s1 = std::min(s0 + 32, n);
                for (uint32_t i = s0; i < s1; i++) out->data[i] = (int8_t)p[i - s0];
                p += 32;
            }
            float total = 0.0f;
            for (uint32_t r = 0; r < b->rows; r++) {
                out->row_scales[r] /= (float)bpr;
                total += out->row_scales[r];
            }
            out->global_scale = total / (float)b->rows;
            return true;
        }
        case 1:  // Q4, Q2, Q1.5: the whole stream decoded from its first byte, scales 1
            if (raw.size() < (size_t)(n + 1) / 2) break;
            dequant_q4_to_int8(raw.data(), out->data.data(), 1.0f, n);
            out->row_scales.assign(b->rows, 1.0f);
            return true;
        case 2:
            if (raw.size() < (size_t)(n + 3) / 4) break;
            dequant_q2_to_int8(raw.data(), out->data.data(), 1.0f, n);
            out->row_scales.assign(b->rows, 1.0f);
            return true;
        case 3:
            if (raw.size() < (size_t)(n + 1) / 2) break;
            dequant_ternary_to_int8(raw.data(), out->data.data(), n);
            out->row_scales.assign(b->rows, 1.0f);
            return true;
        default:
            break;
    }
    *err = "block (" + std::to_string(layer) + ", " + std::to_string(matrix) + ") of type " +
           std::to_string(b->qtype) + " does not decode";
    return false;
}

}  // namespace squeeze
}  // namespace forge
