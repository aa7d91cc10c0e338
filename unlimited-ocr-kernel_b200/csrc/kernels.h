// kernels.h — internal launcher declarations shared by the .cu files and the
// C ABI (capi.cu).  Nothing here is part of the public interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace uocr {

// Device view of one q8-block32 matrix.
struct Q8View {
  const int8_t* w;  // rows*cols
  const float* s;   // rows*ceil(cols/32)
  int rows, cols;
};

// Device view of one SwiGLU FFN (gate/up [width x hidden], down [hidden x width]).
struct FfnView {
  Q8View gate, up, down;
};

// Arithmetic of one projection.
enum Mode : int { MODE_FP32 = 0, MODE_INT8 = 1 };

// q8_elementwise.cu
void launch_dequantize(const int8_t* w, const float* s, int rows, int cols, float* out, int sms,
                       cudaStream_t st);
void launch_quantize_rows(const float* x, long long ld_x, int rows, int cols, int8_t* q, float* s,
                          unsigned* status, int sms, cudaStream_t st);
void launch_validate_q8(const int8_t* w, long long n_w, const float* s, long long n_s,
                        int check_range, unsigned* status, int sms, cudaStream_t st);

// q8_gemv.cu — y[r, :] = W x[r, :] for `batch` rows of x (float, ld_x).
//   MODE_FP32: reordered fp32 accumulation.
//   MODE_INT8: each row block-quantized (into the xq/xs scratch of
//              batch*cols bytes and batch*ceil(cols/32) floats, or in shared
//              memory on the fast path), then the bit-exact ordered
//              accumulation of linear_dynamic_int8.
void launch_gemv(int mode, const Q8View& m, const float* x, long long ld_x, int batch, float* y,
                 long long ld_y, int8_t* xq, float* xs, unsigned* status, int sms,
                 cudaStream_t st);
// Several matrices with the same cols and the same single input row: the
// batched-stream form used to measure GEMV bandwidth (fast path only).
void launch_gemv_multi(int mode, const Q8View* mats, int n, const float* x, float* const* ys,
                       unsigned* status, int sms, cudaStream_t st);
bool gemv_fast_path_ok(const Q8View& m);

// q8_tc.cu — linear_dynamic_int8 for many rows on the tensor cores
// (bit-exact).  Activations are block-quantized rows (launch_quantize_rows):
// xq [rows][cols] int8, xs [rows][cols/32].  Weights: rows % 128 == 0,
// cols % 128 == 0, both arrays 16-byte aligned.
bool q8_tc_supported(int rows, int cols);
size_t q8_tc_maps_bytes();                          // two TMA maps per matrix
bool q8_tc_weight_maps(void* maps, const Q8View& m);  // m's weight and scale maps
cudaError_t launch_q8_tc_single_i8(const Q8View& m, const int8_t* xq, const float* xs, int batch,
                                   float* y, long long ldy, unsigned* status, cudaStream_t st);
// Group g: rows [offsets[g], offsets[g] + counts[g]) of xq/xs times the
// matrix whose q8_tc_weight_maps are maps[g] (device array, 64-byte aligned).
cudaError_t launch_q8_tc_grouped_i8(const void* maps, int groups, const int* counts,
                                    const int* offsets, int max_tiles, int N, int K,
                                    const int8_t* xq, const float* xs, int total_rows, float* y,
                                    long long ldy, unsigned* status, cudaStream_t st);
// Int8Matrix::linear (FP32 activations) for many rows on the tensor cores
// (FP32 tolerance).  Activations come as exact three-way bf16 splits of each
// row scaled by 2^e: pieces [3][rows][cols] and rinv[rows] = 2^-e
// (launch_split_rows / launch_swiglu_split); same weight conditions as the
// int8 kernel.
cudaError_t launch_q8_tc_single_f32(const Q8View& m, const uint16_t* pieces, const float* rinv,
                                    int batch, float* y, long long ldy, unsigned* status,
                                    cudaStream_t st);
cudaError_t launch_q8_tc_grouped_f32(const void* maps, int groups, const int* counts,
                                     const int* offsets, int max_tiles, int N, int K,
                                     const uint16_t* pieces, const float* rinv, int total_rows,
                                     float* y, long long ldy, unsigned* status, cudaStream_t st);
// The row passes below take an optional device row count `live`: rows at or
// past *live are skipped (grouped rows of which only the first *live are in
// use; the pieces keep the stride of `rows`).
// BF16 weights [n][k] (bit patterns) times `batch` FP32 rows given as their
// exact three-way bf16 pieces [3][batch][k] and row scales (launch_split_rows):
// y [batch][ldy], FP32 tolerance (exact products, FP32 accumulation on the
// tensor cores).  k % 64 == 0, weights and pieces 16-byte aligned.
bool linear_bf16_tc_supported(int n, int k);
cudaError_t launch_linear_bf16_tc(const uint16_t* w, int n, int k, const uint16_t* pieces,
                                  const float* rinv, int batch, float* y, long long ldy,
                                  unsigned* status, int sms, cudaStream_t st);
// pieces and rinv of rows x[src ? src[r] : r] (cols % 4 == 0, x rows 16-byte aligned)
void launch_split_rows(const float* x, long long ld_x, const int* src, int rows, int cols,
                       uint16_t* pieces, float* rinv, int sms, cudaStream_t st,
                       const int* live = nullptr);
// pieces and rinv of silu(g) * u
void launch_swiglu_split(const float* g, const float* u, int rows, int cols, uint16_t* pieces,
                         float* rinv, int sms, cudaStream_t st, const int* live = nullptr);
// xq_p[p] = xq[src[p]], xs_p[p] = xs[src[p]]
void launch_gather_rows(const int8_t* xq, const float* xs, const int* src, int rows, int cols,
                        int8_t* xq_p, float* xs_p, int sms, cudaStream_t st,
                        const int* live = nullptr);
// BF16 weights [n][k] (bit patterns) times `batch` float rows of k: the
// reference's sequential BF16 linear (router logits).
cudaError_t launch_linear_bf16(const uint16_t* w, int n, int k, const float* x, int batch, float* y,
                               unsigned* status, cudaStream_t st);
// h = silu(g) * u elementwise (n floats; h may alias g)
void launch_swiglu(const float* g, const float* u, long long n, float* h, int sms, cudaStream_t st);
// acc += the bit patterns of x[0..n) as u64 (the benchmark's logits checksum).
void launch_bits_checksum(const float* x, long long n, unsigned long long* acc, int sms,
                          cudaStream_t st);
// hq/hs = block-quantized silu(g) * u
void launch_swiglu_quantize(const float* g, const float* u, int rows, int cols, int8_t* hq,
                            float* hs, unsigned* status, int sms, cudaStream_t st,
                            const int* live = nullptr);

// q8_small.cu — grouped projections for groups of lo..hi rows (hi <=
// kSmallChunkedMax), as 8-row chunks, weights streamed once per chunk (TMA
// ring), warp-level MMAs over the rows.  int8: xq/xs rows (bit-exact
// linear_dynamic_int8); FP32: pieces [3][piece_rows][K] + rinv (FP32
// tolerance).  Grouped: maps = the groups' q8_tc_weight_maps, rows
// [offsets[g], + counts[g]); `items` (optional) lists the chunks to run
// (group_pairs_kernel writes it; grid.y = max_items).  Single (counts null):
// *single over rows [0, total_rows) in chunks of 8.  maps2 / single2 / y2
// (optional): a second matrix of the same shape over the same rows (gate and
// up in one launch).  x_rows: rows of the int8 activation tensors.
// N % 128 == 0, K % 128 == 0.
constexpr int kSmallRowsMax = 16;
// Grouped launches without a chunk list may take groups of up to this many
// rows, as 8-row chunks (one CTA each, the group's weights re-read from L2);
// with a chunk list, groups of any size.
constexpr int kSmallChunkedMax = 64;
// Upper bound on the 8-row chunks of `pairs` rows in `groups` groups (the
// length of the chunk list group_pairs_kernel writes, without its count).
inline int small_chunk_items(int pairs, int groups) { return (pairs + 7 * groups) / 8 + 1; }
bool small_rows_supported(int N, int K);
cudaError_t launch_small_rows(bool int8, const void* maps, const Q8View* single, const int* counts,
                              const int* offsets, int groups, int lo, int hi, int total_rows, int N,
                              int K, const uint16_t* pieces, int piece_rows, const float* rinv,
                              const int8_t* xq, const float* xs, int x_rows, float* y,
                              long long ldy, unsigned* status, cudaStream_t st,
                              const int* items = nullptr, int max_items = 0,
                              const void* maps2 = nullptr, const Q8View* single2 = nullptr,
                              float* y2 = nullptr);

// moe_route.cu — moe::route for `tokens` rows of logits.  ids/weights are
// tokens*top_k in the reference's order (probability desc, id asc).
void launch_route(const float* logits, int tokens, int n_experts, int top_k, int normalize,
                  float scale, int32_t* ids, float* weights, unsigned* status, int sms,
                  cudaStream_t st);

// moe_decode.cu — one token through Decoder::experts, two PDL-chained kernels.
struct MoeDecodeArgs {
  const FfnView* experts;  // device array [n_experts]
  FfnView shared;
  int n_experts, top_k, normalize;
  float scale;
  int hidden, width, shared_width;
  const float* x;       // [hidden]
  const float* logits;  // [n_experts]
  float* h;             // scratch [shared_width + top_k*width]
  int32_t* route_ids;   // [top_k] (route order)
  float* route_weights; // [top_k]
  float* y;             // [hidden]
  unsigned* status;
  unsigned* grid_sync;  // 4 words, zero before first use, owned by this stream
  // bounded waits: the grid barrier gives up after this many SM cycles (0: the
  // default, about 2 s); barrier_extra > 0 makes it wait for arrivals that
  // never come (host-side fault injection for failure-detection tests)
  long long wait_cycles;
  unsigned barrier_extra;
};
bool moe_decode_supported(const MoeDecodeArgs& a, int sms);
// pdl: allow programmatic dependent launch of the next kernel (off for
// launches captured after a copy node).
cudaError_t launch_moe_decode(int mode, const MoeDecodeArgs& a, int sms, cudaStream_t st,
                              bool pdl = true);

// moe_prefill.cu — many tokens: route, group by expert, grouped projections,
// ordered combine.
struct MoePrefillArgs {
  const FfnView* experts;  // device [n_experts]
  FfnView shared;
  int n_experts, top_k, normalize;
  float scale;
  int hidden, width, shared_width, tokens;
  const float* x;        // [tokens x hidden]
  const float* logits;   // [tokens x n_experts]
  float* y;              // [tokens x hidden]
  int32_t* route_ids;    // [tokens x top_k]
  float* route_weights;  // [tokens x top_k]
  void* workspace;
  size_t workspace_bytes;
  unsigned* status;
  // tensor-core int8 path (optional): [3][n_experts] q8_tc_weight_maps
  // (gate, up, down) in device memory
  const void* tc_maps;
  // Parts of the layer, for callers that split it (expert parallelism):
  // route_given: route_ids/route_weights are inputs (logits unused);
  // skip_shared / skip_routed: leave that part out; pair_out (non-null):
  // the routed outputs, row t*top_k + j for pair (t, j), instead of
  // combining into y.
  int route_given, skip_shared, skip_routed;
  float* pair_out;
  int skip_negative_ids;  // route_given: a negative id marks an unused row
  // optional (0 = tokens): no expert receives more rows than this (a caller
  // whose rows come from several sources of at most this many tokens each
  // selects the kernels by it)
  int max_group_rows;
  // optional (0 = default): groups of up to this many rows run on the
  // warp-level kernel (one CTA per 8-row chunk) when some group can be
  // larger, the rest on the tensor-core GEMMs; the default is kSmallRowsMax
  int small_max;
  // routed part only: leave the expert outputs grouped (no pair_out); read
  // them with moe_prefill_grouped
  int keep_grouped;
  // optional: a second stream (of high priority) and two events; up to
  // kSmallChunkedMax tokens the routing and the routed experts then run on
  // `side` while the shared expert runs on the call's stream (forked after the
  // activations are quantized, joined before the combine)
  cudaStream_t side;
  cudaEvent_t ev_fork, ev_join;
};
size_t moe_prefill_workspace(const MoePrefillArgs& a, int mode);
// The grouped outputs of a keep_grouped call: the output of pair (row) i is
// row token_pos[i] of out_rows (token_pos -1: an unused row).
void moe_prefill_grouped(const MoePrefillArgs& a, int mode, const int** token_pos,
                         const float** out_rows);
cudaError_t launch_moe_prefill(int mode, const MoePrefillArgs& a, int sms, cudaStream_t st);
// Fixed-capacity dispatch for expert parallelism (see moe_prefill.cu).
constexpr int kMaxDispatchRanks = 64;
struct DispatchBounds {
  int world;
  int b[kMaxDispatchRanks + 1];
};
cudaError_t launch_moe_dispatch(const float* x, int tokens, int hidden, const int32_t* ids,
                                int top_k, int n_experts, const int* bounds, int world,
                                int capacity, float* send_x, int32_t* send_ids,
                                int32_t* pair_rows, unsigned* status, cudaStream_t st);
void launch_moe_combine_rows(const int32_t* ids, const float* weights, const float* rows,
                             const int32_t* pair_rows, int tokens, int top_k, int hidden, float* y,
                             cudaStream_t st);
// y[t] += p * out for token t's pairs in ascending expert id (y holds the
// shared expert's output): the combine of Decoder::experts on outputs given
// in pair order (row t*top_k + j).
void launch_moe_combine_pairs(const int32_t* ids, const float* weights, const float* pair_out,
                              int tokens, int top_k, int hidden, float* y, cudaStream_t st);

// attention.cu — decode-side attention ops (RMSNorm, rope, KV cache,
// single-query attention), in the reference's arithmetic order.
// res (optional): normalise sum = x + res instead, written to `sum` (rows of
// ld_x; sum may alias x or res).
void launch_rms_norm(const float* x, long long ld_x, int rows, int width, const float* w, float eps,
                     float* out, long long ld_out, unsigned* status, cudaStream_t st,
                     const float* res = nullptr, float* sum = nullptr);
// table: [max_pos][dim/2] (cos, sin); positions (device, per row) or, when
// null, the cache state {prefix, generated} per row.  b may be null.
void launch_rope(float* a, float* b, long long ld, int rows, int heads, int dim,
                 const int* positions, const int* state, const float2* table, int max_pos,
                 unsigned* status, int sms, cudaStream_t st);
void launch_kv_set_prefix(int* state, int seq, int tokens, cudaStream_t st);
// Device KV cache layouts, per (sequence b, head h) a region of cap x dim
// floats at ((b * heads + h) * cap) * dim:
//   plain: slot-major rows of dim floats;
//   tiled (dim % 32 == 0, cap % 32 == 0): 32-slot tiles of dim/32 blocks of
//     [32 slots][32 floats], so that one tile is one contiguous TMA box of
//     32 x (dim) rows of 128 bytes.
struct KvLayout {
  int heads, dim;
  long long cap;
  int tiled;
};
// LayerCache::push: head h of row b of k/v (token-major, ld floats apart)
// into slot prefix + generated % window of sequence b.
void launch_kv_push(float* keys, float* values, int* state, int batch, const KvLayout& L,
                    int window, const float* k, const float* v, long long ld, unsigned* status,
                    cudaStream_t st);
// Rope of q and k plus the push of k and v, from fused rows [q | k | v].
void launch_kv_rope_push(float* keys, float* values, int* state, int batch, const KvLayout& L,
                         int window, const float* qkv, float* q_out, const float2* table,
                         int max_pos, unsigned* status, cudaStream_t st);
// LayerCache::prefill of sequence seq: token-major rows [tokens][heads*dim].
void launch_kv_prefill(float* keys, float* values, const KvLayout& L, int seq, const float* k,
                       const float* v, int tokens, cudaStream_t st);
// Slots [0, tokens) of sequence seq back as token-major rows.
void launch_kv_export(const float* keys, const float* values, const KvLayout& L, int seq,
                      int tokens, float* k_out, float* v_out, cudaStream_t st);
struct AttnArgs {
  const float* q;  // [batch][ld_q], head h at h * dim
  long long ld_q;
  // Row of token t of head h of sequence b: keys + b * seq_stride +
  // h * head_stride + t * row_stride (same for values).  Token-major
  // ([batch][cap][width], the reference's layout): cap * width, dim, width.
  // Head-major ([batch][heads][cap][dim], the device cache): heads * cap * dim,
  // cap * dim, dim.
  const float* keys;
  const float* values;
  long long seq_stride, head_stride, row_stride;
  long long cap;  // token capacity of a sequence (scores scratch)
  int tiled;      // tiled cache layout (TMA kernel: one box per 32-token tile)
  int width, heads, dim;
  int tokens;          // tokens per sequence when state is null
  const int* state;    // {prefix, generated} per sequence, or null
  // Causal prefill (ops::attention with its mask): the queries are rows
  // 0..batch-1 of the one sequence `seq`, query b at position b over tokens
  // 0..b of that sequence (state and tokens unused).
  int causal, seq;
  // Split form (launch_attention_split): scores scratch [batch][heads][cap].
  float* scores;
  int window;
  float scale;         // 1 / sqrt(dim), as the reference rounds it
  float* out;          // [batch][ld_out]
  long long ld_out;
  unsigned* status;
};
constexpr size_t kAttnMaxSmem = 200 * 1024;
size_t attention_smem_bytes(int dim, int max_tokens);
cudaError_t launch_attention_decode(const AttnArgs& a, int batch, int max_tokens, cudaStream_t st);
// TMA form (head_dim % 32 == 0, <= 256; rows 16-byte aligned): the key and
// value tensor maps of [rows][width] arrays (opaque 128-byte CUtensorMaps).
struct alignas(64) AttnMaps {
  unsigned char k[128];
  unsigned char v[128];
};
// rows x cols: the 2-D view the maps cover ([batch*cap][width] token-major,
// [batch*heads*cap][dim] head-major).
bool attention_tma_ok(const float* keys, const float* values, long long rows, int cols, int dim,
                      long long cap);
bool attention_tma_maps(AttnMaps* m, const float* keys, const float* values, long long rows,
                        int cols);
// Maps of a tiled cache (elements floats per array): box = one 32-slot tile.
bool attention_tma_maps_tiled(AttnMaps* m, const float* keys, const float* values,
                              long long elements, int dim);
// Split form for few sequences (decode, tiled cache, dim % 32 == 0): a scores
// kernel over 128-token chunks, then one kernel per (32-column slice, head,
// sequence) for the softmax and the value sums; the same arithmetic as the
// one-CTA-per-head kernels, so the same bits.  max_tokens bounds every
// sequence's token count (the scratch row length).
bool attention_split_ok(const AttnArgs& a);
// Causal prefill over the tiled cache, 16 query rows per CTA (head_dim 128;
// rows = a.tokens of sequence a.seq; q and out token-major); the same bits as
// the one-query-per-CTA causal form.
bool attention_prefill_ok(const AttnArgs& a);
cudaError_t launch_attention_prefill(const AttnMaps& m, const AttnArgs& a, cudaStream_t st);
cudaError_t launch_attention_split(const AttnArgs& a, int batch, int max_tokens, cudaStream_t st);
cudaError_t launch_attention_decode_tma(const AttnMaps& m, const AttnArgs& a, int batch,
                                        cudaStream_t st);
// rope_table.cpp — host: the reference's cos/sin of every (position, pair).
void build_rope_table(int dim, float theta, int max_pos, float* cos_sin /* [max_pos][dim/2][2] */);

}  // namespace uocr
