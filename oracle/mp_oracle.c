/*
 * CPU oracle for the MiniPrefix paged-KV Llama forward -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is a plain-C restatement of the reference CPU runner's arithmetic
 * (TinyInfer v0.3.0, miniprefix/src/backend/cpu/llama_runner.cpp). Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it, always as the
 * checker. The product path (tinyinfer_b200) never links or calls it.
 *
 * Every function states the reference lines it follows. Summation orders are the
 * reference's own so that, built with -ffp-contract=off, results are bit-identical
 * to the reference CPU runner compiled by oracle/Makefile (pinned in
 * tests/test_oracle_pin.py):
 *   - linear: one accumulator per output element, starting at 0, k ascending,
 *     fused multiply-add for columns inside the 8-wide SIMD blocks and separate
 *     multiply + add for the ragged tail columns
 *     (src/backend/cpu/matmul_kernel.cpp:66-85 AVX2/FMA path, :338-346 tail).
 *   - rms / rope / attention / SwiGLU: the scalar loops of llama_runner.cpp.
 *
 * KV pools use the reference layout [block][layer][slot][kv_width] floats
 * (miniprefix/include/miniprefix/paged_kv.h:25-27, offset formula
 * miniprefix/src/kv/paged_kv.cpp:53-56).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int layers, hidden, intermediate, heads, kv_heads, vocabulary;
    float rms_epsilon, rope_theta;
    int tied;
    int block_tokens;
} oracle_config;

/* Weights in the reference MPFX0001 orientation: every 2-D linear is [in, out]
 * (miniprefix/src/model/model.cpp:28-38); the embedding is [vocab, hidden].
 * Per-layer arrays hold `layers` pointers. lm_head is NULL when tied. */
typedef struct {
    const float* embed;
    const float* final_norm;
    const float* lm_head;
    const float* const* input_norm;
    const float* const* post_norm;
    const float* const* q;
    const float* const* k;
    const float* const* v;
    const float* const* o;
    const float* const* gate;
    const float* const* up;
    const float* const* down;
} oracle_weights;

/* out[r][j] = sum_k x[r][k] * w(k, j), w(k, j) = w[k*w_k + j*w_j].
 * Follows matmul_kernel.cpp:289-354 (run_packed) with the AVX2+FMA micro-kernel
 * :66-85: per element the accumulator starts at 0 and takes k in ascending order;
 * columns below floor(N/8)*8 use fma, the tail uses multiply then add (:338-346). */
void oracle_linear(const float* x, int rows, int inner, const float* w, long w_k, long w_j,
                   int columns, float* out) {
    const int simd_columns = columns - columns % 8;
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (long)r * inner;
        float* o = out + (long)r * columns;
        if (w_j == 1) {
            /* k-outer sweep: each o[j] still takes its k terms in ascending order. */
            for (int j = 0; j < columns; ++j) o[j] = 0.0f;
            for (int k = 0; k < inner; ++k) {
                const float a = xr[k];
                const float* wk = w + k * w_k;
                for (int j = 0; j < simd_columns; ++j) o[j] = fmaf(a, wk[j], o[j]);
                for (int j = simd_columns; j < columns; ++j) {
                    const float p = a * wk[j];
                    o[j] = o[j] + p;
                }
            }
        } else {
            for (int j = 0; j < columns; ++j) {
                float acc = 0.0f;
                const float* wj = w + j * w_j;
                if (j < simd_columns) {
                    for (int k = 0; k < inner; ++k) acc = fmaf(xr[k], wj[k * w_k], acc);
                } else {
                    for (int k = 0; k < inner; ++k) {
                        const float p = xr[k] * wj[k * w_k];
                        acc = acc + p;
                    }
                }
                o[j] = acc;
            }
        }
    }
}

/* RMSNorm: llama_runner.cpp:10-16. */
void oracle_rms(const float* x, int rows, int width, const float* weight, float eps, float* out) {
    for (int r = 0; r < rows; ++r) {
        float sum = 0.0f;
        for (int d = 0; d < width; ++d) {
            const float v = x[(long)r * width + d];
            const float sq = v * v;
            sum = sum + sq;
        }
        const float scale = 1.0f / sqrtf(sum / (float)width + eps);
        for (int d = 0; d < width; ++d) {
            const float t = x[(long)r * width + d] * scale;
            out[(long)r * width + d] = t * weight[d];
        }
    }
}

/* Split-half RoPE in place on x[rows][heads][dim]: llama_runner.cpp:17-22. */
void oracle_rope(float* x, int rows, int heads, int dim, int start, float theta) {
    for (int row = 0; row < rows; ++row)
        for (int h = 0; h < heads; ++h)
            for (int d = 0; d < dim / 2; ++d) {
                const float angle = (float)(start + row) / powf(theta, (float)(2 * d) / (float)dim);
                const float cs = cosf(angle), sn = sinf(angle);
                const long i = ((long)row * heads + h) * dim + d, j = i + dim / 2;
                const float a = x[i], b = x[j];
                const float a_cs = a * cs, b_sn = b * sn, b_cs = b * cs, a_sn = a * sn;
                x[i] = a_cs - b_sn;
                x[j] = b_cs + a_sn;
            }
}

/* Element offset of (layer, token) in one K or V pool: paged_kv.cpp:53-56. */
static long kv_offset(const int* blocks, int block_tokens, int layers, int width, int layer, int token) {
    return (((long)blocks[token / block_tokens] * layers + layer) * block_tokens + token % block_tokens) * width;
}

/* Causal GQA attention for `n` query rows appended at positions used..used+n-1
 * against pages already holding K/V for all used+n tokens: llama_runner.cpp:85-93
 * (naive two-pass softmax; scale = 1/sqrt(dim); kv head = h / (heads/kv_heads)). */
void oracle_attention(const float* q, int n, int used, int heads, int kv_heads, int dim,
                      const float* keys, const float* values, const int* blocks, int block_tokens,
                      int layers, int layer, float* out) {
    const int width = kv_heads * dim;
    const int group = heads / kv_heads;
    float* scores = (float*)malloc(sizeof(float) * (size_t)(used + n));
    const float root = sqrtf((float)dim);
    for (int row = 0; row < n; ++row)
        for (int h = 0; h < heads; ++h) {
            const int length = used + row + 1, kh = h / group;
            float maximum = -INFINITY;
            for (int t = 0; t < length; ++t) {
                const long off = kv_offset(blocks, block_tokens, layers, width, layer, t) + (long)kh * dim;
                float score = 0.0f;
                for (int d = 0; d < dim; ++d) {
                    const float p = q[((long)row * heads + h) * dim + d] * keys[off + d];
                    score = score + p;
                }
                scores[t] = score / root;
                if (scores[t] > maximum) maximum = scores[t];
            }
            float denominator = 0.0f;
            for (int t = 0; t < length; ++t) {
                scores[t] = expf(scores[t] - maximum);
                denominator = denominator + scores[t];
            }
            for (int d = 0; d < dim; ++d) {
                float total = 0.0f;
                for (int t = 0; t < length; ++t) {
                    const long off = kv_offset(blocks, block_tokens, layers, width, layer, t) + (long)kh * dim;
                    const float wgt = scores[t] / denominator;
                    const float p = wgt * values[off + d];
                    total = total + p;
                }
                out[((long)row * heads + h) * dim + d] = total;
            }
        }
    free(scores);
}

/* One append of `n` tokens to a sequence that already holds `used` tokens in
 * `blocks` (which must cover used+n tokens). Writes this append's K/V rows into
 * the pools and the last row's logits. Mirrors CpuRunner::append's arithmetic,
 * llama_runner.cpp:70-101 (the page bookkeeping of :61-69 and :102-103 is the
 * caller's). Returns 0, or 1 when a logit is not finite (:102). */
int oracle_append(const oracle_config* c, const oracle_weights* w, float* keys, float* values,
                  const int* blocks, int used, const int* tokens, int n, float* logits) {
    const int H = c->hidden, I = c->intermediate, dim = H / c->heads, kvw = c->kv_heads * dim;
    float* x = (float*)malloc(sizeof(float) * (size_t)n * H);
    float* normed = (float*)malloc(sizeof(float) * (size_t)n * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)n * H);
    float* k = (float*)malloc(sizeof(float) * (size_t)n * kvw);
    float* v = (float*)malloc(sizeof(float) * (size_t)n * kvw);
    float* ctx = (float*)malloc(sizeof(float) * (size_t)n * H);
    float* proj = (float*)malloc(sizeof(float) * (size_t)n * H);
    float* gate = (float*)malloc(sizeof(float) * (size_t)n * I);
    float* up = (float*)malloc(sizeof(float) * (size_t)n * I);
    for (int r = 0; r < n; ++r) memcpy(x + (long)r * H, w->embed + (long)tokens[r] * H, sizeof(float) * H);
    for (int l = 0; l < c->layers; ++l) {
        oracle_rms(x, n, H, w->input_norm[l], c->rms_epsilon, normed);
        oracle_linear(normed, n, H, w->q[l], H, 1, H, q);
        oracle_linear(normed, n, H, w->k[l], kvw, 1, kvw, k);
        oracle_linear(normed, n, H, w->v[l], kvw, 1, kvw, v);
        oracle_rope(q, n, c->heads, dim, used, c->rope_theta);
        oracle_rope(k, n, c->kv_heads, dim, used, c->rope_theta);
        for (int r = 0; r < n; ++r) {
            const long off = kv_offset(blocks, c->block_tokens, c->layers, kvw, l, used + r);
            memcpy(keys + off, k + (long)r * kvw, sizeof(float) * kvw);
            memcpy(values + off, v + (long)r * kvw, sizeof(float) * kvw);
        }
        oracle_attention(q, n, used, c->heads, c->kv_heads, dim, keys, values, blocks, c->block_tokens,
                         c->layers, l, ctx);
        oracle_linear(ctx, n, H, w->o[l], H, 1, H, proj);
        for (long i = 0; i < (long)n * H; ++i) x[i] = x[i] + proj[i];
        oracle_rms(x, n, H, w->post_norm[l], c->rms_epsilon, normed);
        oracle_linear(normed, n, H, w->gate[l], I, 1, I, gate);
        oracle_linear(normed, n, H, w->up[l], I, 1, I, up);
        for (long i = 0; i < (long)n * I; ++i) {
            const float a = gate[i];
            const float silu = a / (1.0f + expf(-a));
            gate[i] = silu * up[i];
        }
        oracle_linear(gate, n, I, w->down[l], H, 1, H, proj);
        for (long i = 0; i < (long)n * H; ++i) x[i] = x[i] + proj[i];
    }
    oracle_rms(x + (long)(n - 1) * H, 1, H, w->final_norm, c->rms_epsilon, normed);
    if (c->tied) oracle_linear(normed, 1, H, w->embed, 1, H, c->vocabulary, logits);
    else oracle_linear(normed, 1, H, w->lm_head, c->vocabulary, 1, c->vocabulary, logits);
    int bad = 0;
    for (int i = 0; i < c->vocabulary; ++i)
        if (!isfinite(logits[i])) bad = 1;
    free(x); free(normed); free(q); free(k); free(v); free(ctx); free(proj); free(gate); free(up);
    return bad;
}

/* Paged-attention decode operator alone (one query row per sequence, layer 0 of a
 * one-layer pool [block][slot][kv_heads*dim]): the attention loop of
 * llama_runner.cpp:85-93 applied to q[s][heads][dim] against the first lengths[s]
 * tokens addressed through tables[s*table_stride ...]. */
void oracle_decode_attention(const float* q, int sequences, const int* lengths, const int* tables,
                             int table_stride, const float* keys, const float* values, int heads,
                             int kv_heads, int dim, int block_tokens, float* out) {
    for (int s = 0; s < sequences; ++s)
        oracle_attention(q + (long)s * heads * dim, 1, lengths[s] - 1, heads, kv_heads, dim, keys, values,
                         tables + (long)s * table_stride, block_tokens, 1, 0, out + (long)s * heads * dim);
}

/* First index of the maximum (std::max_element), as Engine::step samples:
 * miniprefix/src/engine/engine.cpp:99. */
int oracle_argmax(const float* logits, int count) {
    int best = 0;
    for (int i = 1; i < count; ++i)
        if (logits[i] > logits[best]) best = i;
    return best;
}
