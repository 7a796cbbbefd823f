// mia_layout.h -- the .mia file layout (host code), shared by the writer
// (mia_write.cu) and the model loader (model.cu).
//
// The layout is the one the reference engine reads (src/storage/mia_file.c:
// 41-111) and its converter writes (tools/internal/mia/format.go:129-165):
//   [0, 16384)               112-byte header (mia_header), zero padded
//   [16384, + dense_size)    dense tensors in a fixed order, each at a
//                            64-byte aligned offset: token_embd; per layer
//                            attn_norm, wq, wk, wv, wo, q_norm, k_norm,
//                            ffn_norm, router; output_norm, output.  Matrices
//                            are Q8_0 rows, norms and routers f32.
//   experts_offset (16 KiB)  n_layers * n_experts blobs of expert_blob_size:
//                            gate | up | down, Q8_0, the second and third at
//                            64-byte aligned offsets, the blob 16 KiB aligned
//   tok_offset               the tokenizer bytes
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/miag/miag.h"

namespace miag {

constexpr size_t kMiaHeaderRegion = 16384, kMiaTensorAlign = 64, kMiaExpertAlign = 16384;

inline size_t mia_align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

#pragma pack(push, 1)
struct MiaHeader {  // the on-disk mia_header (include/mia/mia_file.h), 112 bytes
    char magic[4];
    uint32_t version, wtype, dim, n_layers, n_heads, n_kv_heads, head_dim;
    uint32_t vocab, n_experts, n_active, expert_hidden, norm_topk;
    float rope_theta, norm_eps;
    uint32_t pad;
    uint64_t dense_offset, dense_size;
    uint64_t experts_offset, expert_blob_size;
    uint64_t tok_offset, tok_size;
};
#pragma pack(pop)
static_assert(sizeof(MiaHeader) == 112, "mia header");

struct MiaTensor {
    std::string name;
    size_t rows, cols;
    bool quantized;
    size_t offset;  // from the dense section's start
};

inline size_t mia_q8_row_bytes(size_t cols) { return cols / 32 * 36; }

// The dense tensors in the file's order, with their offsets; *total is the
// dense section's size.
inline std::vector<MiaTensor> mia_dense_layout(const miag_mia_config &c, size_t *total) {
    std::vector<MiaTensor> v;
    size_t off = 0;
    auto add = [&](const std::string &name, size_t rows, size_t cols, bool quant) {
        v.push_back({name, rows, cols, quant, off});
        const size_t bytes = quant ? rows * mia_q8_row_bytes(cols) : rows * cols * 4;
        off = mia_align_up(off + bytes, kMiaTensorAlign);
    };
    const size_t d = c.dim, qd = (size_t)c.n_heads * c.head_dim, kvd = (size_t)c.n_kv_heads * c.head_dim;
    add("token_embd", c.vocab, d, true);
    for (uint32_t l = 0; l < c.n_layers; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        add(p + "attn_norm", 1, d, false);
        add(p + "wq", qd, d, true);
        add(p + "wk", kvd, d, true);
        add(p + "wv", kvd, d, true);
        add(p + "wo", d, qd, true);
        add(p + "q_norm", 1, c.head_dim, false);
        add(p + "k_norm", 1, c.head_dim, false);
        add(p + "ffn_norm", 1, d, false);
        add(p + "router", c.n_experts, d, false);
    }
    add("output_norm", 1, d, false);
    add("output", c.vocab, d, true);
    *total = off;
    return v;
}

// Tensors per layer in the dense layout, and the index of each.
constexpr int kMiaLayerTensors = 9;
enum MiaLayerTensor { kAttnNorm, kWq, kWk, kWv, kWo, kQNorm, kKNorm, kFfnNorm, kRouter };
inline size_t mia_layer_tensor(int layer, int which) {
    return 1 + (size_t)layer * kMiaLayerTensors + (size_t)which;
}

// The shapes the writer and the model accept (the reference's limits:
// Q8_0 rows of whole blocks, GQA groups, a NeoX rotation of even length).
inline bool mia_config_ok(const miag_mia_config &c) {
    return c.dim != 0 && c.dim % 32 == 0 && c.expert_hidden != 0 && c.expert_hidden % 32 == 0 &&
           c.n_heads != 0 && c.n_kv_heads != 0 && c.n_heads % c.n_kv_heads == 0 &&
           c.head_dim != 0 && c.head_dim % 2 == 0 && ((size_t)c.n_heads * c.head_dim) % 32 == 0 &&
           c.n_active <= c.n_experts && c.n_layers != 0 && c.vocab != 0;
}

}  // namespace miag
