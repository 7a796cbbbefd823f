// mia_write.cu -- a .mia model file writer (host code), so that models can be
// converted where the reference's Go converter cannot run.
//
// The file is the one the reference engine reads (src/storage/mia_file.c:41-111)
// and its converter writes (tools/internal/mia/format.go:129-165 for the
// layout, :200-263 for the write):
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
// Only one tensor or expert is held at a time.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/miag/miag.h"

namespace {

constexpr size_t kHeaderRegion = 16384, kTensorAlign = 64, kExpertAlign = 16384;

size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

void put_err(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

#pragma pack(push, 1)
struct Header {  // the on-disk mia_header (include/mia/mia_file.h), 112 bytes
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
static_assert(sizeof(Header) == 112, "mia header");

struct Tensor {
    std::string name;
    size_t rows, cols;
    bool quantized;
    size_t offset;  // from the dense section's start
};

size_t q8_row_bytes(size_t cols) { return cols / 32 * 36; }

// The dense tensors in the reference layout's order.
std::vector<Tensor> dense_layout(const miag_mia_config &c, size_t *total) {
    std::vector<Tensor> v;
    size_t off = 0;
    auto add = [&](const std::string &name, size_t rows, size_t cols, bool quant) {
        v.push_back({name, rows, cols, quant, off});
        const size_t bytes = quant ? rows * q8_row_bytes(cols) : rows * cols * 4;
        off = align_up(off + bytes, kTensorAlign);
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

// One row to Q8_0 blocks (the reference quantizer, src/tensor/quant.c:11-27:
// d = amax / 127, id = 1 / d, q = round half away from zero of x * id).
void quantize_row(const float *x, size_t n, unsigned char *out) {
    for (size_t b = 0; b < n / 32; b++) {
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = std::fmax(amax, std::fabs(x[b * 32 + i]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        unsigned char *blk = out + b * 36;
        memcpy(blk, &d, 4);
        for (int i = 0; i < 32; i++) blk[4 + i] = (unsigned char)(int8_t)std::round(x[b * 32 + i] * id);
    }
}

struct Out {
    FILE *f = nullptr;
    uint64_t pos = 0;
    bool ok = true;
    void write(const void *p, size_t n) {
        if (ok && n && fwrite(p, 1, n, f) != n) ok = false;
        pos += n;
    }
    void pad_to(uint64_t off) {
        static const unsigned char zeros[4096] = {0};
        while (ok && pos < off) {
            const size_t n = (size_t)std::min<uint64_t>(sizeof zeros, off - pos);
            write(zeros, n);
        }
    }
};

}  // namespace

extern "C" size_t miag_mia_expert_blob_bytes(const miag_mia_config *c) {
    if (!c) return 0;
    const size_t mat = (size_t)c->expert_hidden * q8_row_bytes(c->dim);
    const size_t up = align_up(mat, kTensorAlign), down = up + align_up(mat, kTensorAlign);
    return align_up(down + (size_t)c->dim * q8_row_bytes(c->expert_hidden), kExpertAlign);
}

extern "C" int miag_mia_write(const char *path, const miag_mia_config *c,
                              miag_mia_dense_source dense, miag_expert_loader expert, void *src_ctx,
                              const void *tokenizer, size_t tokenizer_bytes, char *err,
                              size_t errlen) {
    if (!path || !c || !dense || !expert) {
        put_err(err, errlen, "null argument");
        return -1;
    }
    if (c->dim == 0 || c->dim % 32 || c->expert_hidden == 0 || c->expert_hidden % 32 ||
        c->n_kv_heads == 0 || c->n_heads % c->n_kv_heads || c->head_dim % 2 ||
        ((size_t)c->n_heads * c->head_dim) % 32 || c->n_active > c->n_experts || c->n_layers == 0 ||
        c->vocab == 0) {
        put_err(err, errlen, "unsupported model shape");
        return -1;
    }
    size_t dense_size = 0;
    const std::vector<Tensor> layout = dense_layout(*c, &dense_size);
    Header h;
    memset(&h, 0, sizeof h);
    memcpy(h.magic, "MIA1", 4);
    h.version = 1, h.wtype = 1;  // Q8_0
    h.dim = c->dim, h.n_layers = c->n_layers, h.n_heads = c->n_heads, h.n_kv_heads = c->n_kv_heads;
    h.head_dim = c->head_dim, h.vocab = c->vocab, h.n_experts = c->n_experts;
    h.n_active = c->n_active, h.expert_hidden = c->expert_hidden, h.norm_topk = c->norm_topk;
    h.rope_theta = c->rope_theta, h.norm_eps = c->norm_eps;
    h.dense_offset = kHeaderRegion, h.dense_size = dense_size;
    h.expert_blob_size = miag_mia_expert_blob_bytes(c);
    h.experts_offset = align_up(kHeaderRegion + dense_size, kExpertAlign);
    h.tok_offset = h.experts_offset + (uint64_t)c->n_layers * c->n_experts * h.expert_blob_size;
    h.tok_size = tokenizer ? tokenizer_bytes : 0;

    Out o;
    o.f = fopen(path, "wb");
    if (!o.f) {
        put_err(err, errlen, "open %s for writing failed", path);
        return -1;
    }
    o.write(&h, sizeof h);
    o.pad_to(h.dense_offset);
    std::vector<float> x;
    std::vector<unsigned char> row;
    for (const Tensor &t : layout) {
        x.assign(t.rows * t.cols, 0.0f);
        if (dense(src_ctx, t.name.c_str(), x.data(), x.size()) != 0) {
            put_err(err, errlen, "dense tensor %s: the source failed", t.name.c_str());
            fclose(o.f);
            return -1;
        }
        o.pad_to(h.dense_offset + t.offset);
        if (t.quantized) {
            row.resize(q8_row_bytes(t.cols));
            for (size_t r = 0; r < t.rows; r++) {
                quantize_row(x.data() + r * t.cols, t.cols, row.data());
                o.write(row.data(), row.size());
            }
        } else {
            o.write(x.data(), x.size() * 4);
        }
    }
    std::vector<unsigned char> blob(h.expert_blob_size);
    for (uint32_t l = 0; l < c->n_layers; l++)
        for (uint32_t e = 0; e < c->n_experts; e++) {
            std::fill(blob.begin(), blob.end(), 0);
            if (expert(src_ctx, (int)l, (int)e, blob.data()) != 0) {
                put_err(err, errlen, "expert %u of layer %u: the source failed", e, l);
                fclose(o.f);
                return -1;
            }
            o.pad_to(h.experts_offset + ((uint64_t)l * c->n_experts + e) * h.expert_blob_size);
            o.write(blob.data(), blob.size());
        }
    o.pad_to(h.tok_offset);
    if (tokenizer && tokenizer_bytes) o.write(tokenizer, tokenizer_bytes);
    const bool ok = o.ok && fclose(o.f) == 0;
    if (!ok) {
        put_err(err, errlen, "writing %s failed", path);
        return -1;
    }
    return 0;
}
