// mia_write.cu -- a .mia model file writer (host code), so that models can be
// converted where the reference's Go converter cannot run.
//
// The layout (mia_layout.h) is the one the reference engine reads
// (src/storage/mia_file.c:41-111) and its converter writes
// (tools/internal/mia/format.go:129-165 for the layout, :200-263 for the
// write).
// Only one tensor or expert is held at a time.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "mia_layout.h"

namespace {

using miag::kMiaExpertAlign;
using miag::kMiaHeaderRegion;
using miag::kMiaTensorAlign;
using miag::MiaHeader;
using miag::MiaTensor;
using miag::mia_align_up;
using miag::mia_q8_row_bytes;

void put_err(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
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
    const size_t mat = (size_t)c->expert_hidden * mia_q8_row_bytes(c->dim);
    const size_t up = mia_align_up(mat, kMiaTensorAlign), down = up + mia_align_up(mat, kMiaTensorAlign);
    return mia_align_up(down + (size_t)c->dim * mia_q8_row_bytes(c->expert_hidden), kMiaExpertAlign);
}

extern "C" int miag_mia_write(const char *path, const miag_mia_config *c,
                              miag_mia_dense_source dense, miag_expert_loader expert, void *src_ctx,
                              const void *tokenizer, size_t tokenizer_bytes, char *err,
                              size_t errlen) {
    if (!path || !c || !dense || !expert) {
        put_err(err, errlen, "null argument");
        return -1;
    }
    if (!miag::mia_config_ok(*c)) {
        put_err(err, errlen, "unsupported model shape");
        return -1;
    }
    size_t dense_size = 0;
    const std::vector<MiaTensor> layout = miag::mia_dense_layout(*c, &dense_size);
    MiaHeader h;
    memset(&h, 0, sizeof h);
    memcpy(h.magic, "MIA1", 4);
    h.version = 1, h.wtype = 1;  // Q8_0
    h.dim = c->dim, h.n_layers = c->n_layers, h.n_heads = c->n_heads, h.n_kv_heads = c->n_kv_heads;
    h.head_dim = c->head_dim, h.vocab = c->vocab, h.n_experts = c->n_experts;
    h.n_active = c->n_active, h.expert_hidden = c->expert_hidden, h.norm_topk = c->norm_topk;
    h.rope_theta = c->rope_theta, h.norm_eps = c->norm_eps;
    h.dense_offset = kMiaHeaderRegion, h.dense_size = dense_size;
    h.expert_blob_size = miag_mia_expert_blob_bytes(c);
    h.experts_offset = mia_align_up(kMiaHeaderRegion + dense_size, kMiaExpertAlign);
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
    for (const MiaTensor &t : layout) {
        x.assign(t.rows * t.cols, 0.0f);
        if (dense(src_ctx, t.name.c_str(), x.data(), x.size()) != 0) {
            put_err(err, errlen, "dense tensor %s: the source failed", t.name.c_str());
            fclose(o.f);
            return -1;
        }
        o.pad_to(h.dense_offset + t.offset);
        if (t.quantized) {
            row.resize(mia_q8_row_bytes(t.cols));
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
