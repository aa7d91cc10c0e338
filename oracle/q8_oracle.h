/*
 * q8_oracle.h — CPU restatement of the reference's q8-block32 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker or the timed CPU baseline.  The product path
 * (libuocr_q8.so) never links or calls it.
 *
 * Every function restates the reference's *portable scalar* Rust path (the
 * branch it runs on x86-64 Linux: no NEON, no Accelerate), file:line cited
 * beside each declaration.  Arithmetic contract:
 *   - compiled with -ffp-contract=off -fno-fast-math (Rust never fuses a*b+c);
 *   - every float sum is strictly left-to-right and starts at -0.0f, the
 *     neutral element of Rust's `impl Sum for f32`;
 *   - round-half-to-even via rintf() under the default rounding mode;
 *   - exp via the platform libm expf(), as Rust's f32::exp lowers to it.
 *
 * Parity pins: the reference's own known answers (tests/quantized_loader.rs:
 * 41-48, tests/moe.rs:5-10), its bit-exact and tolerance tests
 * (tests/quantized.rs), the four-row bit-equality patterns (src/cpu/neon.rs:
 * 245-276) and vectors produced by the reference's importable Python quantizer
 * (tools/quantize.py:19-34) committed under tests/golden/.
 */
#ifndef Q8_ORACLE_H
#define Q8_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: one per OcrError variant (src/error.rs:1-17). */
enum {
  Q8O_OK = 0,
  Q8O_IO = 1,
  Q8O_JSON = 2,
  Q8O_FORMAT = 3,
  Q8O_SHAPE = 4,
  Q8O_UNSUPPORTED = 5,
  Q8O_RESOURCE = 6,
  Q8O_NUMERICAL = 7
};

/* Projection dispatch (src/decoder/mod.rs:99-112).
 *   Q8O_WEIGHTS_ONLY    : Int8Matrix::linear for every batch.
 *   Q8O_DYNAMIC         : linear_dynamic_int8 when the input has exactly one
 *                         row, linear otherwise (the reference's rule).
 *   Q8O_DYNAMIC_ROWWISE : extension for M>1 — linear_dynamic_int8 applied to
 *                         each row independently. */
enum { Q8O_WEIGHTS_ONLY = 0, Q8O_DYNAMIC = 1, Q8O_DYNAMIC_ROWWISE = 2 };

typedef struct {
  size_t rows, cols;
  const int8_t *w; /* rows*cols, row-major */
  const float *s;  /* rows*ceil(cols/32) */
} q8o_mat;

typedef struct {
  q8o_mat gate, up, down;
} q8o_ffn;

/* Worker threads used by the row-parallel loops (like rayon's pool; row
 * partitioning never changes per-row arithmetic).  n<=0 -> all cores. */
void q8o_set_threads(int n);
int q8o_get_threads(void);

/* Int8Matrix::from_parts validation (src/cpu/quantized.rs:18-42). */
int q8o_from_parts_check(size_t rows, size_t cols, size_t weights_len, size_t scales_len,
                         const float *scales);

/* Int8Matrix::quantize (src/cpu/quantized.rs:43-74).  Also the activation
 * quantizer of linear_dynamic_int8 (:169). */
int q8o_quantize(size_t rows, size_t cols, const float *x, int8_t *w, float *s);

/* Int8Matrix::dequantize (src/cpu/quantized.rs:75-95). */
void q8o_dequantize(size_t rows, size_t cols, const int8_t *w, const float *s, float *out);

/* Int8Matrix::linear (src/cpu/quantized.rs:99-149; batch!=1 branch via
 * ops::linear, src/cpu/ops.rs:39-47 — the same arithmetic).  x is
 * batch*cols, y is batch*rows. */
int q8o_linear(const q8o_mat *m, const float *x, size_t batch, float *y);

/* Int8Matrix::linear_dynamic_int8 (src/cpu/quantized.rs:155-236), single row. */
int q8o_linear_dynamic_int8(const q8o_mat *m, const float *x, float *y);

/* Row-wise extension of linear_dynamic_int8 to batch rows. */
int q8o_linear_dynamic_int8_rows(const q8o_mat *m, const float *x, size_t batch, float *y);

/* Block sums S_b of linear_dynamic_int8 for one output row (exact int32),
 * exposed so tests can check the integer stage separately. */
void q8o_block_sums(const int8_t *w, const int8_t *xq, size_t cols, int32_t *sums);

/* ops::softmax scalar path (src/cpu/ops.rs:135-187). */
int q8o_softmax(float *v, size_t n);

/* moe::route (src/decoder/moe.rs:7-30).  Writes `count` (id, weight) pairs in
 * the reference's order: probability descending, expert id ascending. */
int q8o_route(const float *logits, size_t n, size_t count, int normalize, float scale,
              int32_t *ids, float *weights);

/* ops::silu (src/cpu/ops.rs:225-229). */
void q8o_silu(float *v, size_t n);

/* ops::linear_weight BF16 branch (src/cpu/ops.rs:62-133): router GEMV.
 * w_bf16 is n*k little-endian bf16 bit patterns; x is batch*k. */
int q8o_linear_bf16(const uint16_t *w_bf16, size_t n, size_t k, const float *x, size_t batch,
                    float *y);

/* Decoder::feed_forward (src/decoder/mod.rs:114-122) under a dispatch mode. */
int q8o_feed_forward(const q8o_ffn *f, const float *x, size_t rows, int mode, float *out);

/* Decoder::experts (src/decoder/mod.rs:124-220) given router logits
 * (tokens*n_experts).  Shared expert first, then routed experts in ascending
 * id, result[row] += p*out.  sel_ids / sel_weights (tokens*top_k, optional)
 * receive each token's selection in route() order. */
int q8o_experts(const q8o_ffn *shared, const q8o_ffn *experts, size_t n_experts,
                const float *logits, const float *x, size_t tokens, size_t hidden, size_t top_k,
                int normalize, float scale, int mode, float *out, int32_t *sel_ids,
                float *sel_weights);

/* ops::rms_norm (src/cpu/ops.rs:362-414, 419-421): rows x width. */
int q8o_rms_norm(const float *x, size_t rows, size_t width, const float *weight, float eps,
                 float *out);

/* ops::rope (src/cpu/ops.rs:423-437): every head of `values` (n floats) at
 * one position, in place. */
int q8o_rope(float *values, size_t n, size_t head_dim, size_t position, float theta);

/* ops::attention_decode (src/cpu/ops.rs:515-606), scalar branch: q of width
 * floats over token-major keys/values of keys_len floats each. */
int q8o_attention_decode(const float *q, size_t width, const float *keys, size_t keys_len,
                         const float *values, size_t values_len, size_t heads, float *out);

/* ops::attention (src/cpu/ops.rs:263-360), scalar branch: q [heads][nq][dim]
 * over k, v [heads][nk][dim]; causal (nq == nk) masks the keys after each
 * query's own position. */
int q8o_attention(const float *q, size_t heads, size_t nq, size_t dim, const float *k,
                  const float *v, size_t nk, int causal, float *out);

#ifdef __cplusplus
}
#endif
#endif
