/*
 * q8_oracle.c — CPU restatement of the reference's q8-block32 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see q8_oracle.h).  Compile with
 *   gcc -O2 -ffp-contract=off -fno-fast-math -pthread
 * so that no product/sum is contracted into an FMA and no denormal is
 * flushed; the reference's Rust never does either.
 */
#include "q8_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define BLOCK 32

static int g_threads = 0;

void q8o_set_threads(int n) { g_threads = n; }

int q8o_get_threads(void) {
  if (g_threads > 0) return g_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* Row-parallel loop, like rayon's par_iter over output rows: each worker owns
 * a contiguous row range, so per-row arithmetic is independent of the thread
 * count. */
typedef void (*row_fn)(void *ctx, size_t r0, size_t r1);
typedef struct {
  row_fn fn;
  void *ctx;
  size_t r0, r1;
} row_task;

static void *row_worker(void *arg) {
  row_task *t = (row_task *)arg;
  t->fn(t->ctx, t->r0, t->r1);
  return NULL;
}

static void parallel_rows(size_t rows, row_fn fn, void *ctx) {
  int nt = q8o_get_threads();
  if (nt > 256) nt = 256;
  if ((size_t)nt > rows) nt = (int)rows;
  if (nt <= 1 || rows < 64) {
    fn(ctx, 0, rows);
    return;
  }
  pthread_t th[256];
  row_task tasks[256];
  int started[256] = {0};
  for (int i = 0; i < nt; ++i) {
    tasks[i].fn = fn;
    tasks[i].ctx = ctx;
    tasks[i].r0 = rows * (size_t)i / (size_t)nt;
    tasks[i].r1 = rows * (size_t)(i + 1) / (size_t)nt;
    if (i > 0) started[i] = pthread_create(&th[i], NULL, row_worker, &tasks[i]) == 0;
  }
  fn(ctx, tasks[0].r0, tasks[0].r1);
  for (int i = 1; i < nt; ++i) {
    if (started[i])
      pthread_join(th[i], NULL);
    else
      fn(ctx, tasks[i].r0, tasks[i].r1);
  }
}

static size_t blocks_of(size_t cols) { return (cols + BLOCK - 1) / BLOCK; }

static int mul_overflows(size_t a, size_t b, size_t *out) {
  if (a != 0 && b > SIZE_MAX / a) return 1;
  *out = a * b;
  return 0;
}

/* src/cpu/quantized.rs:24-35 */
int q8o_from_parts_check(size_t rows, size_t cols, size_t weights_len, size_t scales_len,
                         const float *scales) {
  size_t n, ns;
  if (rows == 0 || cols == 0 || mul_overflows(rows, cols, &n) || n != weights_len ||
      mul_overflows(rows, blocks_of(cols), &ns) || ns != scales_len)
    return Q8O_SHAPE;
  for (size_t i = 0; i < scales_len; ++i)
    if (!isfinite(scales[i]) || scales[i] < 0.0f) return Q8O_NUMERICAL;
  return Q8O_OK;
}

/* src/cpu/quantized.rs:43-74: per 32-column block, max = fold(0, max)(|v|),
 * scale = max / 127 (IEEE f32 division), q = clamp(rint(v / scale), -127, 127),
 * or 0 for an all-zero block; nonfinite input and scale underflow are
 * Numerical errors. */
int q8o_quantize(size_t rows, size_t cols, const float *x, int8_t *w, float *s) {
  size_t n;
  if (rows == 0 || cols == 0 || mul_overflows(rows, cols, &n)) return Q8O_SHAPE;
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(x[i])) return Q8O_NUMERICAL;
  const size_t nb = blocks_of(cols);
  for (size_t r = 0; r < rows; ++r) {
    const float *row = x + r * cols;
    for (size_t b = 0; b < nb; ++b) {
      const size_t c0 = b * BLOCK, c1 = c0 + BLOCK < cols ? c0 + BLOCK : cols;
      float max = 0.0f;
      for (size_t c = c0; c < c1; ++c) max = fmaxf(max, fabsf(row[c]));
      const float scale = max / 127.0f;
      if (max > 0.0f && scale == 0.0f) return Q8O_NUMERICAL;
      s[r * nb + b] = scale;
      for (size_t c = c0; c < c1; ++c) {
        int8_t q = 0;
        if (scale != 0.0f) {
          float v = rintf(row[c] / scale);
          if (v < -127.0f) v = -127.0f;
          if (v > 127.0f) v = 127.0f;
          q = (int8_t)v;
        }
        w[r * cols + c] = q;
      }
    }
  }
  return Q8O_OK;
}

/* src/cpu/quantized.rs:75-95: one f32 product, one rounding. */
typedef struct {
  size_t cols;
  const int8_t *w;
  const float *s;
  float *out;
} deq_ctx;

static void deq_rows(void *p, size_t r0, size_t r1) {
  const deq_ctx *c = (const deq_ctx *)p;
  const size_t nb = blocks_of(c->cols);
  for (size_t r = r0; r < r1; ++r)
    for (size_t k = 0; k < c->cols; ++k)
      c->out[r * c->cols + k] = (float)c->w[r * c->cols + k] * c->s[r * nb + k / BLOCK];
}

void q8o_dequantize(size_t rows, size_t cols, const int8_t *w, const float *s, float *out) {
  deq_ctx c = {cols, w, s, out};
  parallel_rows(rows, deq_rows, &c);
}

/* One output of Int8Matrix::linear, scalar branch (src/cpu/quantized.rs:126-130):
 * sum of ((w as f32) * scale) * x, left to right from -0.0. */
static float dot_fp32(const int8_t *w, const float *s, const float *x, size_t cols) {
  float acc = -0.0f;
  for (size_t k = 0; k < cols; ++k) acc += (float)w[k] * s[k / BLOCK] * x[k];
  return acc;
}

/* src/cpu/quantized.rs:99-149.  The batch!=1 branch dequantizes and runs
 * ops::linear (src/cpu/ops.rs:39-47): sum of x * fl(w*s) from -0.0, which is
 * the same sequence of roundings as the batch==1 branch. */
typedef struct {
  const q8o_mat *m;
  const float *x;
  size_t batch;
  float *y;
} lin_ctx;

static void lin_rows(void *p, size_t r0, size_t r1) {
  const lin_ctx *c = (const lin_ctx *)p;
  const size_t cols = c->m->cols, nb = blocks_of(cols);
  for (size_t i = 0; i < c->batch; ++i)
    for (size_t r = r0; r < r1; ++r)
      c->y[i * c->m->rows + r] =
          dot_fp32(c->m->w + r * cols, c->m->s + r * nb, c->x + i * cols, cols);
}

int q8o_linear(const q8o_mat *m, const float *x, size_t batch, float *y) {
  lin_ctx c = {m, x, batch, y};
  parallel_rows(m->rows, lin_rows, &c);
  return Q8O_OK;
}

void q8o_block_sums(const int8_t *w, const int8_t *xq, size_t cols, int32_t *sums) {
  const size_t nb = blocks_of(cols);
  for (size_t b = 0; b < nb; ++b) {
    const size_t c0 = b * BLOCK, c1 = c0 + BLOCK < cols ? c0 + BLOCK : cols;
    int32_t acc = 0;
    for (size_t c = c0; c < c1; ++c) acc += (int32_t)w[c] * (int32_t)xq[c];
    sums[b] = acc;
  }
}

/* One output of linear_dynamic_int8, scalar branch (src/cpu/quantized.rs:190-198):
 * exact int32 block sums S_b, then sum of ((S_b as f32) * ws[b]) * xs[b]
 * from -0.0, block order, no FMA. */
static float dot_int8(const int8_t *w, const float *ws, const int8_t *xq, const float *xs,
                      size_t cols) {
  const size_t nb = blocks_of(cols);
  float acc = -0.0f;
  for (size_t b = 0; b < nb; ++b) {
    const size_t c0 = b * BLOCK, c1 = c0 + BLOCK < cols ? c0 + BLOCK : cols;
    int32_t sum = 0;
    for (size_t c = c0; c < c1; ++c) sum += (int32_t)w[c] * (int32_t)xq[c];
    acc += (float)sum * ws[b] * xs[b];
  }
  return acc;
}

typedef struct {
  const q8o_mat *m;
  const int8_t *xq;
  const float *xs;
  float *y;
} dyn_ctx;

static void dyn_rows(void *p, size_t r0, size_t r1) {
  const dyn_ctx *c = (const dyn_ctx *)p;
  const size_t cols = c->m->cols, nb = blocks_of(cols);
  for (size_t r = r0; r < r1; ++r)
    c->y[r] = dot_int8(c->m->w + r * cols, c->m->s + r * nb, c->xq, c->xs, cols);
}

static int dynamic_row(const q8o_mat *m, const float *x, float *y) {
  const size_t nb = blocks_of(m->cols);
  int8_t *xq = (int8_t *)malloc(m->cols);
  float *xs = (float *)malloc(nb * sizeof(float));
  if (!xq || !xs) {
    free(xq);
    free(xs);
    return Q8O_RESOURCE;
  }
  int st = q8o_quantize(1, m->cols, x, xq, xs); /* src/cpu/quantized.rs:169 */
  if (st == Q8O_OK) {
    dyn_ctx c = {m, xq, xs, y};
    parallel_rows(m->rows, dyn_rows, &c);
  }
  free(xq);
  free(xs);
  return st;
}

int q8o_linear_dynamic_int8(const q8o_mat *m, const float *x, float *y) {
  return dynamic_row(m, x, y);
}

int q8o_linear_dynamic_int8_rows(const q8o_mat *m, const float *x, size_t batch, float *y) {
  for (size_t i = 0; i < batch; ++i) {
    int st = dynamic_row(m, x + i * m->cols, y + i * m->rows);
    if (st) return st;
  }
  return Q8O_OK;
}

/* src/cpu/ops.rs:135-187, scalar branch: reject NaN/+inf, max must be finite,
 * subtract, expf, sequential sum from -0.0, divide. */
int q8o_softmax(float *v, size_t n) {
  if (n == 0) return Q8O_NUMERICAL;
  for (size_t i = 0; i < n; ++i)
    if (isnan(v[i]) || v[i] == INFINITY) return Q8O_NUMERICAL;
  float maximum = -INFINITY;
  for (size_t i = 0; i < n; ++i) maximum = fmaxf(maximum, v[i]);
  if (!isfinite(maximum)) return Q8O_NUMERICAL;
  for (size_t i = 0; i < n; ++i) v[i] -= maximum;
  for (size_t i = 0; i < n; ++i) v[i] = expf(v[i]);
  float sum = -0.0f;
  for (size_t i = 0; i < n; ++i) sum += v[i];
  for (size_t i = 0; i < n; ++i) v[i] /= sum;
  return Q8O_OK;
}

typedef struct {
  int32_t id;
  float p;
} pick;

/* b.1.total_cmp(&a.1).then(a.0.cmp(&b.0)) for nonnegative, non-NaN values. */
static int pick_cmp(const void *a, const void *b) {
  const pick *x = (const pick *)a, *y = (const pick *)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  if (signbit(x->p) != signbit(y->p)) return signbit(x->p) ? 1 : -1;
  return x->id < y->id ? -1 : (x->id > y->id);
}

/* src/decoder/moe.rs:7-30 */
int q8o_route(const float *logits, size_t n, size_t count, int normalize, float scale,
              int32_t *ids, float *weights) {
  if (count == 0 || count > n || !isfinite(scale) || scale <= 0.0f) return Q8O_SHAPE;
  float *p = (float *)malloc(n * sizeof(float));
  pick *order = (pick *)malloc(n * sizeof(pick));
  if (!p || !order) {
    free(p);
    free(order);
    return Q8O_RESOURCE;
  }
  memcpy(p, logits, n * sizeof(float));
  int st = q8o_softmax(p, n);
  if (st == Q8O_OK) {
    for (size_t i = 0; i < n; ++i) {
      order[i].id = (int32_t)i;
      order[i].p = p[i];
    }
    qsort(order, n, sizeof(pick), pick_cmp);
    float denominator = 1.0f;
    if (normalize) {
      float sum = -0.0f;
      for (size_t i = 0; i < count; ++i) sum += order[i].p;
      denominator = sum + 1e-20f;
    }
    for (size_t i = 0; i < count; ++i) {
      ids[i] = order[i].id;
      weights[i] = order[i].p / denominator * scale;
    }
  }
  free(p);
  free(order);
  return st;
}

/* src/cpu/ops.rs:225-229 */
void q8o_silu(float *v, size_t n) {
  for (size_t i = 0; i < n; ++i) v[i] /= 1.0f + expf(-v[i]);
}

static float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* src/cpu/ops.rs:62-133 (BF16 branch; the multi-row branch converts to f32
 * and runs ops::linear, the same per-output arithmetic). */
int q8o_linear_bf16(const uint16_t *w, size_t n, size_t k, const float *x, size_t batch,
                    float *y) {
  if (n == 0 || k == 0) return Q8O_SHAPE;
  for (size_t i = 0; i < batch; ++i)
    for (size_t r = 0; r < n; ++r) {
      float acc = -0.0f;
      for (size_t c = 0; c < k; ++c) acc += bf16_to_f32(w[r * k + c]) * x[i * k + c];
      y[i * n + r] = acc;
    }
  return Q8O_OK;
}

/* Decoder::projection (src/decoder/mod.rs:99-112) for an overlay hit. */
static int projection(const q8o_mat *m, const float *x, size_t rows, int mode, float *y) {
  if (mode == Q8O_DYNAMIC && rows == 1) return q8o_linear_dynamic_int8(m, x, y);
  if (mode == Q8O_DYNAMIC_ROWWISE) return q8o_linear_dynamic_int8_rows(m, x, rows, y);
  return q8o_linear(m, x, rows, y);
}

/* src/decoder/mod.rs:114-122 */
int q8o_feed_forward(const q8o_ffn *f, const float *x, size_t rows, int mode, float *out) {
  const size_t width = f->gate.rows;
  float *gate = (float *)malloc(rows * width * sizeof(float));
  float *up = (float *)malloc(rows * width * sizeof(float));
  int st = (!gate || !up) ? Q8O_RESOURCE : Q8O_OK;
  if (!st) st = projection(&f->gate, x, rows, mode, gate);
  if (!st) st = projection(&f->up, x, rows, mode, up);
  if (!st) {
    q8o_silu(gate, rows * width);
    for (size_t i = 0; i < rows * width; ++i) gate[i] *= up[i];
    st = projection(&f->down, gate, rows, mode, out);
  }
  free(gate);
  free(up);
  return st;
}

/* src/decoder/mod.rs:124-220.  Both of the reference's branches (parallel
 * decode tasks and the serial grouped loop) add p*out to the shared expert's
 * output in ascending expert id, so one loop restates both. */
int q8o_experts(const q8o_ffn *shared, const q8o_ffn *experts, size_t n_experts,
                const float *logits, const float *x, size_t tokens, size_t hidden, size_t top_k,
                int normalize, float scale, int mode, float *out, int32_t *sel_ids,
                float *sel_weights) {
  int32_t *ids = (int32_t *)malloc(tokens * top_k * sizeof(int32_t));
  float *wts = (float *)malloc(tokens * top_k * sizeof(float));
  size_t *rows = (size_t *)malloc(tokens * sizeof(size_t));
  float *probs = (float *)malloc(tokens * sizeof(float));
  float *gathered = (float *)malloc(tokens * hidden * sizeof(float));
  float *result = (float *)malloc(tokens * hidden * sizeof(float));
  int st = (!ids || !wts || !rows || !probs || !gathered || !result) ? Q8O_RESOURCE : Q8O_OK;
  for (size_t t = 0; !st && t < tokens; ++t)
    st = q8o_route(logits + t * n_experts, n_experts, top_k, normalize, scale, ids + t * top_k,
                   wts + t * top_k);
  if (!st) st = q8o_feed_forward(shared, x, tokens, mode, out);
  for (size_t e = 0; !st && e < n_experts; ++e) {
    size_t count = 0;
    for (size_t t = 0; t < tokens; ++t)
      for (size_t j = 0; j < top_k; ++j)
        if ((size_t)ids[t * top_k + j] == e) {
          rows[count] = t;
          probs[count] = wts[t * top_k + j];
          ++count;
        }
    if (!count) continue;
    for (size_t i = 0; i < count; ++i)
      memcpy(gathered + i * hidden, x + rows[i] * hidden, hidden * sizeof(float));
    st = q8o_feed_forward(&experts[e], gathered, count, mode, result);
    for (size_t i = 0; !st && i < count; ++i) {
      float *dest = out + rows[i] * hidden;
      const float *src = result + i * hidden;
      for (size_t c = 0; c < hidden; ++c) dest[c] += probs[i] * src[c];
    }
  }
  if (!st && sel_ids) memcpy(sel_ids, ids, tokens * top_k * sizeof(int32_t));
  if (!st && sel_weights) memcpy(sel_weights, wts, tokens * top_k * sizeof(float));
  free(ids);
  free(wts);
  free(rows);
  free(probs);
  free(gathered);
  free(result);
  return st;
}

/* src/cpu/ops.rs:362-414 with center = false (rms_norm, :419-421): shape
 * checks, nonfinite input or weight -> Numerical, then per row the squares
 * summed left to right from -0.0, divided by the width, sqrt, reciprocal,
 * and (x - 0) * scale * w + 0 per element. */
int q8o_rms_norm(const float *x, size_t rows, size_t width, const float *weight, float eps,
                 float *out) {
  if (width == 0 || !isfinite(eps) || eps <= 0.0f) return Q8O_SHAPE;
  for (size_t i = 0; i < rows * width; ++i)
    if (!isfinite(x[i])) return Q8O_NUMERICAL;
  for (size_t i = 0; i < width; ++i)
    if (!isfinite(weight[i])) return Q8O_NUMERICAL;
  for (size_t r = 0; r < rows; ++r) {
    const float *in = x + r * width;
    float *o = out + r * width;
    const float mean = 0.0f;
    float variance = -0.0f;
    for (size_t i = 0; i < width; ++i) variance += (in[i] - mean) * (in[i] - mean);
    variance /= (float)width;
    const float scale = 1.0f / sqrtf(variance + eps);
    for (size_t i = 0; i < width; ++i) o[i] = (in[i] - mean) * scale * weight[i] + 0.0f;
  }
  return Q8O_OK;
}

/* src/cpu/ops.rs:423-437 */
int q8o_rope(float *values, size_t n, size_t head_dim, size_t position, float theta) {
  if (head_dim == 0 || head_dim % 2 || n % head_dim || !isfinite(theta) || theta <= 0.0f)
    return Q8O_SHAPE;
  const size_t half = head_dim / 2;
  for (size_t h = 0; h < n; h += head_dim) {
    float *head = values + h;
    for (size_t i = 0; i < half; ++i) {
      const float angle = (float)position / powf(theta, 2.0f * (float)i / (float)head_dim);
      const float s = sinf(angle), c = cosf(angle);
      const float a = head[i], b = head[i + half];
      head[i] = a * c - b * s;
      head[i + half] = b * c + a * s;
    }
  }
  return Q8O_OK;
}

/* src/cpu/ops.rs:515-606, scalar branch (one head after another): per head
 * the token scores (left-to-right dot from -0.0, times 1/sqrt(dim)), the
 * softmax, then out[d] += score * value over the tokens in order. */
int q8o_attention_decode(const float *q, size_t width, const float *keys, size_t keys_len,
                         const float *values, size_t values_len, size_t heads, float *out) {
  if (heads == 0 || width == 0 || width % heads || keys_len == 0 || keys_len % width ||
      keys_len != values_len)
    return Q8O_SHAPE;
  const size_t tokens = keys_len / width, dim = width / heads;
  const float scale = 1.0f / sqrtf((float)dim);
  float *scores = (float *)malloc(tokens * sizeof(float));
  if (!scores) return Q8O_RESOURCE;
  for (size_t i = 0; i < width; ++i) out[i] = 0.0f;
  for (size_t h = 0; h < heads; ++h) {
    const size_t off = h * dim;
    for (size_t t = 0; t < tokens; ++t) {
      float acc = -0.0f;
      for (size_t d = 0; d < dim; ++d) acc += q[off + d] * keys[t * width + off + d];
      scores[t] = acc;
    }
    for (size_t t = 0; t < tokens; ++t) scores[t] *= scale;
    int st = q8o_softmax(scores, tokens);
    if (st) {
      free(scores);
      return st;
    }
    for (size_t t = 0; t < tokens; ++t)
      for (size_t d = 0; d < dim; ++d) out[off + d] += scores[t] * values[t * width + off + d];
  }
  free(scores);
  return Q8O_OK;
}

/* ops::attention (src/cpu/ops.rs:263-360) with its causal mask
 * (softmax_rows, :190-222), scalar branch: q [heads][nq][dim] over k, v
 * [heads][nk][dim].  Per head and query row i: scores over all nk keys
 * (left-to-right dot from -0.0, times 1/sqrt(dim)); when causal (nq == nk)
 * the scores after key i become -inf; the softmax; then each output element
 * is the left-to-right sum from -0.0 over all nk keys of score * value (the
 * masked keys add products of +0.0).  The reference's query blocks change
 * only how many rows are held at once, not a row's arithmetic. */
int q8o_attention(const float *q, size_t heads, size_t nq, size_t dim, const float *k,
                  const float *v, size_t nk, int causal, float *out) {
  if (heads == 0 || nq == 0 || nk == 0 || dim == 0 || (causal && nq != nk)) return Q8O_SHAPE;
  const float scale = 1.0f / sqrtf((float)dim);
  float *scores = (float *)malloc(nk * sizeof(float));
  if (!scores) return Q8O_RESOURCE;
  for (size_t h = 0; h < heads; ++h) {
    const float *kh = k + h * nk * dim, *vh = v + h * nk * dim;
    for (size_t i = 0; i < nq; ++i) {
      const float *qi = q + (h * nq + i) * dim;
      for (size_t t = 0; t < nk; ++t) {
        float acc = -0.0f;
        for (size_t d = 0; d < dim; ++d) acc += qi[d] * kh[t * dim + d];
        scores[t] = acc;
      }
      for (size_t t = 0; t < nk; ++t) scores[t] *= scale;
      if (causal)
        for (size_t t = i + 1; t < nk; ++t) scores[t] = -INFINITY;
      int st = q8o_softmax(scores, nk);
      if (st) {
        free(scores);
        return st;
      }
      float *o = out + (h * nq + i) * dim;
      for (size_t d = 0; d < dim; ++d) {
        float acc = -0.0f;
        for (size_t t = 0; t < nk; ++t) acc += scores[t] * vh[t * dim + d];
        o[d] = acc;
      }
    }
  }
  free(scores);
  return Q8O_OK;
}
