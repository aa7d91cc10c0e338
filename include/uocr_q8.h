/*
 * uocr_q8.h — C ABI of the B200 q8-block32 quantized matrix-product path.
 *
 * Drop-in boundary for the reference runtime's INT8 block-32 operator surface
 * (ezgamehost/unlimited-ocr-kernel, Rust crate `uocr`).  The reference has no
 * FFI of its own: each entry point below replaces the Rust method cited beside
 * it, with the same argument meaning and the same error variants.  All
 * signatures use plain pointers and sizes.  `stream` arguments are
 * cudaStream_t values passed as void* (NULL = the context's stream).
 *
 * Storage format (src/cpu/quantized.rs:9-16; overlay contract
 * docs/benchmarks/2026-09-28-int8-kernels/README.md "uocr-q8-block32-v1"):
 * row-major int8 weights [rows x cols] and one float32 scale per 32
 * consecutive columns of a row, [rows x ceil(cols/32)]; the last block of a
 * row may be short.  Dequantized weight = (float)w * scale.
 *
 * Arithmetic contract:
 *   - DYNAMIC (int8-activation) results are bit-identical to the reference's
 *     scalar path: activation block quantization (IEEE division, round half
 *     to even), exact int32 block dots, and the ordered per-block float
 *     accumulation of linear_dynamic_int8 (src/cpu/quantized.rs:190-198).
 *   - WEIGHTS_ONLY (FP32-activation) results reorder the float accumulation;
 *     max relative error <= 1e-4 of max(|y|, sum|w'x| * 2^-10).
 *   - dequantize and quantize are bit-identical.
 *
 * Error convention: every function returns a uocr_status; uocr_last_error()
 * returns the calling thread's last message.  Input errors detected on the
 * device (nonfinite activations, scale underflow, invalid router rows) do not
 * trap: they are recorded in the context and returned by the next
 * synchronising call (uocr_ctx_sync, or any *_host function).
 *
 * Threading: a context is used by one host thread at a time (the reference's
 * `&mut CpuContext`, src/cpu/mod.rs:68-71); matrices and MoE layers are
 * immutable after creation and may be shared by contexts on the same device.
 */
#ifndef UOCR_Q8_H
#define UOCR_Q8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UOCR_Q8_BLOCK 32
#define UOCR_Q8_ABI_VERSION 1

/* One code per OcrError variant (src/error.rs:1-17) plus device codes. */
typedef enum uocr_status {
  UOCR_OK = 0,
  UOCR_ERR_IO = 1,          /* OcrError::Io */
  UOCR_ERR_JSON = 2,        /* OcrError::Json */
  UOCR_ERR_FORMAT = 3,      /* OcrError::Format */
  UOCR_ERR_SHAPE = 4,       /* OcrError::Shape */
  UOCR_ERR_UNSUPPORTED = 5, /* OcrError::Unsupported */
  UOCR_ERR_RESOURCE = 6,    /* OcrError::Resource */
  UOCR_ERR_NUMERICAL = 7,   /* OcrError::Numerical */
  UOCR_ERR_CUDA = 8,        /* CUDA runtime error */
  UOCR_ERR_NCCL = 9,        /* NCCL error (expert-parallel exchange) */
  UOCR_ERR_TIMEOUT = 10,    /* a bounded device wait expired */
  UOCR_ERR_INVALID = 11     /* null handle / pointer */
} uocr_status;

/* QuantizationMode (src/cpu/quantized.rs:242-247) and the row-wise
 * extension.  Decoder::projection (src/decoder/mod.rs:99-112) uses int8
 * activations only for a single-row input in DynamicActivations mode. */
typedef enum uocr_mode {
  UOCR_WEIGHTS_ONLY = 0,          /* QuantizationMode::WeightsOnly */
  UOCR_DYNAMIC_ACTIVATIONS = 1,   /* QuantizationMode::DynamicActivations */
  UOCR_DYNAMIC_ROWWISE = 2        /* int8 activations for every row (extension) */
} uocr_mode;

typedef struct uocr_ctx uocr_ctx;
typedef struct uocr_q8 uocr_q8;
typedef struct uocr_moe uocr_moe;

/* ---- library ------------------------------------------------------------ */
int uocr_abi_version(void);
const char *uocr_last_error(void);
const char *uocr_status_name(int status);

/* ---- context: CpuContext::new (src/cpu/mod.rs:26-49) ---------------------
 * device: CUDA ordinal.  scratch_limit: bytes, the reference's scratch_limit
 * (0 -> Resource error, like threads/scratch 0 in CpuContext::new); every
 * operation applies the reference's check_elements rule (count*4 > limit ->
 * Resource, src/cpu/mod.rs:73-78) with the reference's element counts. */
int uocr_ctx_create(int device, size_t scratch_limit, uocr_ctx **out);
int uocr_ctx_destroy(uocr_ctx *ctx);
int uocr_ctx_set_stream(uocr_ctx *ctx, void *stream);
/* Wait for the context's stream; return and clear device-detected errors. */
int uocr_ctx_sync(uocr_ctx *ctx);
int uocr_ctx_device(const uocr_ctx *ctx, int *device, int *sm_count);
/* No counterpart in the reference (which has no device waits).  The bounded
 * device waits of the context's kernels (the one-token decode kernel's grid
 * barrier) give up after `ns` nanoseconds (0: the default, about 2 s) and
 * report UOCR_ERR_TIMEOUT at the next synchronising call. */
int uocr_ctx_set_wait_limit(uocr_ctx *ctx, uint64_t ns);
/* Failure-detection test hook, host-side (no GPU fault): while `hold` is
 * nonzero, the one-token decode kernel's grid barrier waits for one arrival
 * more than its grid makes, so every such launch runs out its wait limit and
 * the next synchronising call reports UOCR_ERR_TIMEOUT.  The barrier's words
 * stay valid: after the hold is cleared the next launch is exact again. */
int uocr_ctx_hold_decode_barrier(uocr_ctx *ctx, int hold);

/* ---- matrices: Int8Matrix (src/cpu/quantized.rs:11-237) -----------------
 * Int8Matrix::from_parts (:18-42): copies host weights/scales to the device.
 * Shape if rows/cols is 0 or a length disagrees; Numerical if a scale is
 * NaN, infinite or negative (-0.0 is accepted). */
int uocr_q8_from_parts(uocr_ctx *ctx, size_t rows, size_t cols, const int8_t *weights,
                       size_t weights_len, const float *scales, size_t scales_len,
                       uocr_q8 **out);
/* Same validation for device-resident storage; the handle borrows (does not
 * free) the memory.  Scale validation runs on the device and is reported
 * synchronously.  Like Int8Matrix, the matrix is immutable: the memory must
 * not be written while the handle lives (the one-token MoE kernel starts
 * streaming weights before the previous kernel in the stream has finished). */
int uocr_q8_from_device(uocr_ctx *ctx, size_t rows, size_t cols, const int8_t *weights_dev,
                        const float *scales_dev, uocr_q8 **out);
/* Int8Matrix::quantize (:43-74) of a host float matrix, on the device. */
int uocr_q8_quantize(uocr_ctx *ctx, size_t rows, size_t cols, const float *values,
                     uocr_q8 **out);
int uocr_q8_free(uocr_q8 *m);
int uocr_q8_shape(const uocr_q8 *m, size_t *rows, size_t *cols);
/* Int8Matrix::storage_bytes (:96-98). */
size_t uocr_q8_storage_bytes(const uocr_q8 *m);
int uocr_q8_device_ptrs(const uocr_q8 *m, const int8_t **weights_dev, const float **scales_dev);
int uocr_q8_download(uocr_ctx *ctx, const uocr_q8 *m, int8_t *weights, float *scales);

/* Int8Matrix::dequantize (:75-95): out_dev is rows*cols floats. */
int uocr_q8_dequantize(uocr_ctx *ctx, const uocr_q8 *m, float *out_dev);
int uocr_q8_dequantize_host(uocr_ctx *ctx, const uocr_q8 *m, float *out, size_t out_len);

/* Int8Matrix::linear (:99-149): y[r, :] = W x[r, :] for `batch` rows.
 * Device buffers, asynchronous on the context stream. */
int uocr_q8_linear(uocr_ctx *ctx, const uocr_q8 *m, const float *x_dev, size_t batch,
                   float *y_dev);
/* Host tensors like the reference: x has shape x_shape[0..ndim) whose last
 * extent must equal cols (Shape otherwise); y receives the same shape with
 * the last extent replaced by rows.  Synchronous. */
int uocr_q8_linear_host(uocr_ctx *ctx, const uocr_q8 *m, const float *x, const size_t *x_shape,
                        size_t ndim, float *y, size_t y_len);

/* Int8Matrix::linear_dynamic_int8 (:155-236).  Device form: each of `batch`
 * rows is quantized and multiplied independently (row-wise extension; batch
 * 1 is the reference operation). */
int uocr_q8_linear_dynamic_int8(uocr_ctx *ctx, const uocr_q8 *m, const float *x_dev,
                                size_t batch, float *y_dev);
/* Host form with the reference's rule: exactly one input row, else Shape. */
int uocr_q8_linear_dynamic_int8_host(uocr_ctx *ctx, const uocr_q8 *m, const float *x,
                                     const size_t *x_shape, size_t ndim, float *y,
                                     size_t y_len);

/* Block quantization of `rows` float rows on the device (the activation step
 * of linear_dynamic_int8, :169): q_dev rows*cols int8, s_dev
 * rows*ceil(cols/32) floats. */
int uocr_q8_quantize_rows(uocr_ctx *ctx, const float *x_dev, size_t rows, size_t cols,
                          int8_t *q_dev, float *s_dev);

/* Several matrices of equal cols applied to one shared input row, one launch
 * (the batched-stream GEMV; all experts of a token share their input). */
int uocr_q8_linear_multi(uocr_ctx *ctx, const uocr_q8 *const *mats, size_t n, int mode,
                         const float *x_dev, float *const *y_dev);

/* ---- routing: moe::route (src/decoder/moe.rs:7-30) -----------------------
 * logits_dev tokens*n_experts; ids_dev/weights_dev tokens*top_k in the
 * reference's order (probability descending, expert id ascending).  Shape if
 * top_k == 0, top_k > n_experts or scale is not finite and > 0; Numerical if
 * a row holds NaN/+inf or no finite maximum (ops::softmax). */
int uocr_moe_route(uocr_ctx *ctx, const float *logits_dev, size_t tokens, size_t n_experts,
                   size_t top_k, int normalize, float scale, int32_t *ids_dev,
                   float *weights_dev);

/* ---- MoE layer: Decoder::experts (src/decoder/mod.rs:124-220) ------------
 * shared_*: the fused shared-expert FFN (width n_shared*moe_intermediate);
 * gate/up/down: n_experts routed FFNs.  All gate/up are [width x hidden],
 * down [hidden x width].  The layer keeps the handles' device pointers; the
 * matrices must outlive it. */
int uocr_moe_create(uocr_ctx *ctx, const uocr_q8 *shared_gate, const uocr_q8 *shared_up,
                    const uocr_q8 *shared_down, const uocr_q8 *const *gate,
                    const uocr_q8 *const *up, const uocr_q8 *const *down, size_t n_experts,
                    size_t top_k, int normalize_topk, float routed_scale, uocr_moe **out);
int uocr_moe_free(uocr_moe *layer);
/* One MoE FFN over `tokens` rows: x_dev tokens*hidden, router logits
 * tokens*n_experts, y_dev tokens*hidden.  ids/weights (optional, may be
 * NULL) receive each token's routing.  mode: uocr_mode.  Asynchronous.
 * Between 2 and 64 tokens the routing and the routed experts run on a second,
 * high-priority stream owned by the context while the shared expert runs on
 * the context's stream; the second stream is forked from and joined back into
 * the context's stream within the call (events), so the call stays ordered on
 * that stream and can be captured in a CUDA graph. */
int uocr_moe_forward(uocr_ctx *ctx, const uocr_moe *layer, int mode, const float *x_dev,
                     const float *logits_dev, size_t tokens, float *y_dev, int32_t *ids_dev,
                     float *weights_dev);
/* Host-buffer form: copies in, runs, copies out, synchronises. */
int uocr_moe_forward_host(uocr_ctx *ctx, const uocr_moe *layer, int mode, const float *x,
                          const float *logits, size_t tokens, float *y, int32_t *ids,
                          float *weights);

/* ---- expert parallelism: uocr_moe_forward in parts ------------------------
 * No counterpart in the reference: Decoder::experts (src/decoder/mod.rs:
 * 124-220) runs every expert where the tokens are.  A caller that places the
 * routed experts of a layer on several GPUs splits the forward into
 *   uocr_moe_route        routing of this GPU's tokens (ids, weights)
 *   uocr_moe_expert_rows  the experts this GPU holds, applied to rows sent
 *                         to it (each with its expert id local to `layer`)
 *   uocr_moe_shared_rows  the shared expert over this GPU's tokens, into y
 *   uocr_moe_combine      y[t] += weight * expert output, ascending expert id
 * and moves rows between GPUs itself.  With the routed rows of each expert
 * applied in one uocr_moe_expert_rows call per source GPU (in
 * UOCR_DYNAMIC_ACTIVATIONS an expert's row count selects its arithmetic), the
 * result is uocr_moe_forward's on this GPU's tokens, bit for bit.  A layer
 * made for these calls holds only its own experts; its top_k and routing
 * arguments are not used by them.  All asynchronous on the context stream. */
/* out_dev[i] = FFN_{expert_ids_dev[i]}(x_dev[i]): x_dev/out_dev rows*hidden.
 * Rows of one expert form one group, as the tokens an expert receives in
 * Decoder::experts.  A negative id marks an unused row (a padding slot of
 * uocr_moe_dispatch): it is skipped and its output row left unchanged.  An
 * id >= n_experts is Shape at the next synchronising call. */
int uocr_moe_expert_rows(uocr_ctx *ctx, const uocr_moe *layer, int mode, const float *x_dev,
                         const int32_t *expert_ids_dev, size_t rows, float *out_dev);
/* y_dev = shared FFN(x_dev), rows*hidden each. */
int uocr_moe_shared_rows(uocr_ctx *ctx, const uocr_moe *layer, int mode, const float *x_dev,
                         size_t rows, float *y_dev);
/* Fixed-capacity dispatch, so that the exchange needs no counts on the host
 * (and a whole expert-parallel step can be captured in a CUDA graph): pair
 * (t, j) goes to the rank r with rank_bounds[r] <= ids[t,j] <
 * rank_bounds[r+1] (rank_bounds: host array of world + 1 increasing expert
 * indices from 0), in slot s = the number of earlier pairs for r;
 * send_x[r][s] = x[t], send_ids[r][s] = ids[t,j] - rank_bounds[r] (-1 in
 * unused slots), pair_rows[t*top_k + j] = r * capacity + s.  send_x is
 * world*capacity*hidden floats, send_ids world*capacity.  More than
 * `capacity` pairs for one rank is Resource at the next synchronising call
 * (tokens * top_k always suffices).  world <= 64, top_k <= 8, hidden % 4 == 0. */
int uocr_moe_dispatch(uocr_ctx *ctx, const float *x_dev, size_t tokens, size_t hidden,
                      const int32_t *ids_dev, size_t top_k, const int32_t *rank_bounds,
                      size_t world, size_t capacity, float *send_x_dev, int32_t *send_ids_dev,
                      int32_t *pair_rows_dev);
/* uocr_moe_combine with the expert outputs read at rows_dev[pair_rows[t*top_k
 * + j]] (the returned fixed-capacity buffer of uocr_moe_dispatch). */
int uocr_moe_combine_rows(uocr_ctx *ctx, const int32_t *ids_dev, const float *weights_dev,
                          const float *rows_dev, const int32_t *pair_rows_dev, size_t tokens,
                          size_t top_k, size_t hidden, float *y_dev);
/* For each token t: y[t] += weights[t,j] * pair_out[t*top_k + j] over its
 * top_k pairs in ascending ids[t,j], one rounding per operation (the combine
 * of src/decoder/mod.rs:208-217; y holds the shared output).  top_k <= 8. */
int uocr_moe_combine(uocr_ctx *ctx, const int32_t *ids_dev, const float *weights_dev,
                     const float *pair_out_dev, size_t tokens, size_t top_k, size_t hidden,
                     float *y_dev);

/* ---- expert parallelism over NVLink peer memory ----------------------------
 * No counterpart in the reference (Decoder::experts, src/decoder/mod.rs:
 * 124-220, runs on one device).  A layer whose routed experts are split over
 * `world` GPUs of one node in contiguous blocks (rank r holds experts
 * [rank_bounds[r], rank_bounds[r+1]) as `local_layer`, every rank holds the
 * shared expert and brings its own tokens).  Rows travel as stores into the
 * other GPUs' memory (CUDA IPC mappings; no collective library, no padding,
 * no host synchronisation): a step is capturable in a CUDA graph, and its
 * result on each rank is uocr_moe_forward of that rank's tokens: routing and
 * int8-activation outputs bit for bit; FP32-activation outputs within the
 * FP32 tolerance (an owner's group, rows of several ranks, may take another
 * projection kernel, with another FP32 summation order).
 *
 *   uocr_ep_create   this rank's end: device buffers for up to max_tokens
 *                    tokens per rank and step (the same on every rank).
 *   uocr_ep_handle   UOCR_EP_HANDLE_BYTES describing this rank's buffers
 *                    (a CUDA IPC handle); the caller gathers all ranks'
 *                    handles by any channel (MPI, a TCP store, ...) and
 *   uocr_ep_connect  opens them (world * UOCR_EP_HANDLE_BYTES, rank order).
 *                    Ranks in one process (testing several ranks on one GPU)
 *                    use uocr_ep_connect_local instead.
 *   uocr_ep_forward  one step of this rank's tokens, asynchronous on the
 *                    context's stream (the exchange runs on an internal
 *                    high-priority stream forked from and joined back into
 *                    it).  Every rank must run the same number of steps, in
 *                    the same order; a rank with no tokens passes tokens = 0.
 *   uocr_ep_dispatch / uocr_ep_experts / uocr_ep_combine: the same step in
 *                    three parts on the context's stream, for one host thread
 *                    driving several ranks of one process on ONE stream in
 *                    the order dispatch(all ranks), experts(all ranks),
 *                    combine(all ranks), so that no wait depends on work
 *                    queued behind it.
 * Every device wait is bounded (uocr_ep_set_wait_limit, default 2 s); a wait
 * that expires returns UOCR_ERR_TIMEOUT at the next synchronising call, after
 * which the layers of all ranks must be freed and created again.  tokens >
 * max_tokens is Resource; x_dev and y_dev 16-byte aligned; hidden % 4 == 0;
 * world <= 64, top_k <= 8, n_experts <= 256. */
typedef struct uocr_ep uocr_ep;
#define UOCR_EP_HANDLE_BYTES 128
int uocr_ep_create(uocr_ctx *ctx, const uocr_moe *local_layer, size_t n_experts, size_t top_k,
                   int normalize_topk, float routed_scale, const int32_t *rank_bounds,
                   size_t world, size_t rank, size_t max_tokens, uocr_ep **out);
int uocr_ep_free(uocr_ep *ep);
int uocr_ep_handle(const uocr_ep *ep, void *handle_out);
int uocr_ep_connect(uocr_ep *ep, const void *handles);
int uocr_ep_connect_local(uocr_ep *const *eps, size_t world);
int uocr_ep_set_wait_limit(uocr_ep *ep, uint64_t ns);
int uocr_ep_forward(uocr_ctx *ctx, uocr_ep *ep, int mode, const float *x_dev,
                    const float *logits_dev, size_t tokens, float *y_dev, int32_t *ids_dev,
                    float *weights_dev);
/* Host-buffer form of uocr_ep_forward (x tokens*hidden, logits
 * tokens*n_experts, y tokens*hidden floats): copies in, one step, copies out,
 * synchronises and returns the step's device status (pinned buffers are
 * copied directly, others through a pinned mirror). */
int uocr_ep_forward_host(uocr_ctx *ctx, uocr_ep *ep, int mode, const float *x,
                         const float *logits, size_t tokens, float *y);
int uocr_ep_dispatch(uocr_ctx *ctx, uocr_ep *ep, int mode, const float *x_dev,
                     const float *logits_dev, size_t tokens, float *y_dev);
int uocr_ep_experts(uocr_ctx *ctx, uocr_ep *ep);
int uocr_ep_combine(uocr_ctx *ctx, uocr_ep *ep, float *y_dev, int32_t *ids_dev,
                    float *weights_dev);

/* ---- allocation-free decode ------------------------------------------------
 * No counterpart in the reference.  For callers that may not allocate device
 * memory while inference runs (a serving loop that reserves everything at
 * start-up, a host whose pool allocator owns all device memory): the same
 * one-token MoE FFN as uocr_moe_forward(tokens = 1), bit-identical results,
 * but it calls no cudaMalloc/cudaFree.  Its scratch is a fixed array inside
 * the library (UOCR_NOALLOC_MAX_H floats for h, plus the routing), held by
 * every GPU that loads the library until the process exits; layers needing
 * more are rejected with UOCR_ERR_RESOURCE, layers outside the single-token
 * decode kernels with UOCR_ERR_UNSUPPORTED.  The first call on a device looks
 * up the array's device address (make it before any stream capture).  All
 * calls on a device share the array: calls that overlap on the GPU race, so
 * serialise them.  The array's address is cached per device for the life of
 * the process: do not use the library across a cudaDeviceReset of a device it
 * has served.  x_dev hidden floats (16-byte aligned), logits_dev
 * n_experts floats, y_dev hidden floats; asynchronous on the context stream. */
#define UOCR_NOALLOC_MAX_H 16384
int uocr_moe_forward_decode_noalloc(uocr_ctx *ctx, const uocr_moe *layer, int mode,
                                    const float *x_dev, const float *logits_dev, float *y_dev);

/* Decoder::feed_forward (src/decoder/mod.rs:114-122): y = down(silu(gate x) *
 * (up x)) for `rows` rows of x_dev (device, gate->cols floats each; y_dev rows
 * of down->rows floats).  Each projection's arithmetic follows
 * Decoder::projection (:99-112): int8 activations for a one-row input in
 * UOCR_DYNAMIC_ACTIVATIONS, for every row in UOCR_DYNAMIC_ROWWISE (rows of
 * independent sequences at decode), FP32 activations otherwise.  Shape when
 * gate/up/down disagree; asynchronous on the context's stream. */
int uocr_feed_forward(uocr_ctx *ctx, const uocr_q8 *gate, const uocr_q8 *up, const uocr_q8 *down,
                      int mode, const float *x_dev, size_t rows, float *y_dev);

/* ops::linear_weight, BF16 branch (src/cpu/ops.rs:62-133): y [batch x n] = x
 * [batch x k] (device floats) times a BF16 weight [n x k] (device bit
 * patterns), each output a left-to-right float sum as in the reference (bit
 * for bit): the router logits of Decoder::experts ("mlp.gate.weight" is not
 * in the INT8 overlay).  Sized for router-like n; asynchronous. */
int uocr_linear_bf16(uocr_ctx *ctx, const uint16_t *w_dev, size_t n, size_t k, const float *x_dev,
                     size_t batch, float *y_dev);
/* The same product for large BF16 weights (the lm_head, n = 129,280): each
 * row of x is split into three bf16 pieces that sum to it exactly, so every
 * product on the tensor cores is exact, and the sums accumulate in FP32 in
 * another order than the reference's (FP32 tolerance, as Int8Matrix::linear
 * on the tensor cores).  Streams the BF16 weights at HBM rate.  k % 64 == 0;
 * w_dev and x_dev 16-byte aligned; asynchronous. */
int uocr_linear_bf16_tc(uocr_ctx *ctx, const uint16_t *w_dev, size_t n, size_t k,
                        const float *x_dev, size_t batch, float *y_dev);

/* ---- decoder attention at decode --------------------------------------------
 * The attention half of Decoder::layer (src/decoder/mod.rs:241-341) for one
 * new token per sequence, on device pointers, asynchronous on the context's
 * stream.  Arithmetic follows the reference's order (sequential sums, one
 * rounding per operation); results equal the reference's bit for bit
 * except where exp rounds differently (rarely one ulp of a softmax weight).
 * Input errors found on the device (nonfinite norm input, a position past the
 * rotary table, a cache used before its prefill) are reported at the next
 * synchronising call, as for the other entry points. */
typedef struct uocr_rope uocr_rope;
typedef struct uocr_kv uocr_kv;

/* The fixed-work decoder benchmark's logits checksum (src/model/benchmark.rs:
 * 43-47): *acc_dev (device u64) += the bit pattern of each of the n floats
 * of x_dev, wrapping modulo 2^64, so equal to the reference's sequential
 * wrapping_add.  Asynchronous on the context's stream. */
int uocr_bits_checksum(uocr_ctx *ctx, const float *x_dev, size_t n, uint64_t *acc_dev);

/* ops::rms_norm (src/cpu/ops.rs:362-414,419-421): rows x width, weight of
 * width floats; out may equal x.  Shape for width 0 or eps not finite and
 * positive; Numerical ("normalization") for a nonfinite input or weight. */
int uocr_rms_norm(uocr_ctx *ctx, const float *x_dev, size_t rows, size_t width,
                  const float *weight_dev, float eps, float *out_dev);
/* The residual add of Decoder::layer (src/decoder/mod.rs:348-349, 361-362)
 * fused with the RMSNorm that follows it (:355, or the next layer's input
 * norm): sum = x + res elementwise (one rounding each; sum may equal x or
 * res), out = rms_norm(sum), bit-identical to the add followed by
 * uocr_rms_norm.  No reference entry point of its own; errors as
 * uocr_rms_norm. */
int uocr_add_rms_norm(uocr_ctx *ctx, const float *x_dev, const float *res_dev, size_t rows,
                      size_t width, const float *weight_dev, float eps, float *sum_dev,
                      float *out_dev);

/* ops::rope (src/cpu/ops.rs:423-437): a table of cos/sin for positions
 * [0, max_positions), built on the host with the reference's single-precision
 * operations; uocr_rope_apply rotates q (and k unless NULL) in place, rows x
 * width in heads of head_dim, row r at positions_dev[r] (int32).  A position
 * outside the table is Resource ("maximum context exceeded"). */
int uocr_rope_create(uocr_ctx *ctx, size_t head_dim, float theta, size_t max_positions,
                     uocr_rope **out);
int uocr_rope_free(uocr_rope *rope);
int uocr_rope_apply(uocr_ctx *ctx, const uocr_rope *rope, float *q_dev, float *k_dev, size_t rows,
                    size_t width, const int32_t *positions_dev);

/* ops::attention_decode (src/cpu/ops.rs:515-606): one query q [1 x width]
 * over token-major keys/values (keys_len = values_len = tokens * width),
 * heads of width/heads; out [width].  Same layout and scratch checks. */
int uocr_attention_decode(uocr_ctx *ctx, const float *q_dev, const float *keys_dev,
                          size_t keys_len, const float *values_dev, size_t values_len,
                          size_t width, size_t heads, float *out_dev);

/* The prefill branch of Decoder::layer (src/decoder/mod.rs:313-338): causal
 * ops::attention (src/cpu/ops.rs:263-360, its mask in softmax_rows :190-222)
 * of token-major q, keys, values [tokens x width] in heads of width/heads;
 * out [tokens x width], row i over tokens 0..i.  The same arithmetic order as
 * the reference's, so row i equals uocr_attention_decode over tokens 0..i; the
 * outputs match the reference bit for bit except where exp rounds differently
 * and in the sign of an output that is zero.  Shape for an empty or uneven
 * layout; Resource under the reference's scratch rule (dim*tokens +
 * tokens*width + tokens elements); Unsupported beyond 65535 tokens. */
int uocr_attention_prefill(uocr_ctx *ctx, const float *q_dev, const float *keys_dev,
                           const float *values_dev, size_t tokens, size_t width, size_t heads,
                           float *out_dev);

/* LayerCache (src/decoder/cache.rs) for `batch` sequences on the device: an
 * immutable prefix of up to max_prefix tokens followed by a ring of `window`
 * tokens (slot of a new token: prefix + generated % window).  Stored per
 * (sequence, head) so that a head's tokens stream contiguously (for head_dim
 * a multiple of 32, in 32-slot tiles that are one contiguous 16 KB-class
 * block each); a head's slot order is the reference's physical token order.
 * Inputs (prefill rows, pushed k/v) and uocr_kv_export's output are
 * token-major rows of heads * head_dim floats, as in the reference.  The per-sequence counters live in device memory, so
 * push, rope and attention can be captured in CUDA graphs.
 *   uocr_kv_prefill: LayerCache::prefill of sequence seq (device rows);
 *   uocr_kv_push:    LayerCache::push of row b of k/v ([batch x width]) into
 *                    every sequence b;
 *   uocr_kv_rope:    ops::rope of q and k rows at each sequence's position
 *                    (before this token's push);
 *   uocr_kv_attention: ops::attention_decode of q row b over sequence b;
 *   uocr_kv_attention_prefill: the causal attention of a prefill
 *                    (uocr_attention_prefill) of q rows [rows x width] of
 *                    sequence seq over its prefix, right after
 *                    uocr_kv_prefill of those rows (Shape unless rows equals
 *                    that prefix);
 *   uocr_kv_state:   LayerCache::tokens and ::position (synchronous);
 *   uocr_kv_export:  LayerCache::keys / ::values of sequence seq as
 *                    token-major rows (device; NULL outputs: *tokens only).
 *   uocr_kv_reset:   sequence seq empty again (LayerCache::new), to be
 *                    prefilled anew;
 * push / rope / attention before every sequence is prefilled: Shape. */
int uocr_kv_create(uocr_ctx *ctx, size_t batch, size_t heads, size_t head_dim, size_t window,
                   size_t max_prefix, uocr_kv **out);
int uocr_kv_free(uocr_kv *kv);
int uocr_kv_reset(uocr_ctx *ctx, uocr_kv *kv, size_t seq);
/* The form uocr_kv_attention runs: 0 (default) chooses by size, 1 one CTA per
 * (head, sequence), 2 split over tokens (a scores kernel over token chunks,
 * then per head-dimension slice the softmax and value sums; caches whose
 * head_dim is a multiple of 32 only, else Unsupported).  Every form gives
 * the same bits; the choice only moves time. */
int uocr_kv_set_attention_form(uocr_kv *kv, int form);
int uocr_kv_prefill(uocr_ctx *ctx, uocr_kv *kv, size_t seq, const float *keys_dev,
                    const float *values_dev, size_t tokens);
int uocr_kv_push(uocr_ctx *ctx, uocr_kv *kv, const float *k_dev, const float *v_dev);
int uocr_kv_rope(uocr_ctx *ctx, const uocr_kv *kv, const uocr_rope *rope, float *q_dev,
                 float *k_dev);
int uocr_kv_attention(uocr_ctx *ctx, const uocr_kv *kv, const float *q_dev, float *out_dev);
int uocr_kv_attention_prefill(uocr_ctx *ctx, const uocr_kv *kv, size_t seq, const float *q_dev,
                              size_t rows, float *out_dev);
/* uocr_kv_rope then uocr_kv_push in one launch, reading the fused q/k/v
 * projection rows [q | k | v] (batch x 3*heads*head_dim, device): q is rotated
 * into q_out_dev (batch x heads*head_dim), k rotated and v copied into the
 * cache.  Same results as the two calls. */
int uocr_kv_rope_push_qkv(uocr_ctx *ctx, uocr_kv *kv, const uocr_rope *rope, const float *qkv_dev,
                          float *q_out_dev);
int uocr_kv_state(uocr_ctx *ctx, const uocr_kv *kv, size_t seq, size_t *tokens, size_t *position);
int uocr_kv_export(uocr_ctx *ctx, const uocr_kv *kv, size_t seq, float *keys_out,
                   float *values_out, size_t *tokens);

/* ---- INT8 overlay (QuantizedWeights) --------------------------------------
 * The "uocr-q8-block32-v1" overlay: a safetensors file holding, for every
 * projection matrix of the source checkpoint, "<name>" (I8 [rows, cols]) and
 * "<name>.q8_scales" (F32 [rows, ceil(cols/32)]), next to a JSON manifest at
 * the overlay path with its extension replaced by ".json".
 *
 * uocr_overlay_load replaces QuantizedWeights::load(path, &source)
 * (src/cpu/quantized.rs:304-362): overlay_path is `path`, source_path the
 * file behind `source` (Checkpoint::open, src/checkpoint.rs:101-166, whose
 * checks it also applies).  Every check of the reference runs on the host in
 * the reference's order with its error variant: manifest (Io, Json),
 * safetensors layout (Format, Json), version and metadata, SHA-256 of the
 * source and of the overlay, the set of eligible matrices, per matrix dtype /
 * shape / no byte -128 (Format), then Int8Matrix::from_parts (Shape,
 * Numerical).  A valid overlay is uploaded into one device allocation on the
 * context's device (each array 256-byte aligned); nothing is allocated for
 * an invalid one.  Synchronous.
 *
 * uocr_overlay_check: the same validation without a device (no upload);
 * optional outputs: the matrix count and the device bytes a load takes.
 *
 * uocr_overlay_get replaces QuantizedWeights::get (quantized.rs:363-365):
 * *out = the matrix named `name`, or NULL when the overlay has none (returns
 * UOCR_OK either way).  The handle belongs to the overlay: do not free it;
 * it is valid until uocr_overlay_free.  Names enumerate in byte order.
 *
 * uocr_sha256_file: lowercase hex SHA-256 of a file (65 bytes with the NUL),
 * the digest the manifest records (tools/fetch_model.py sha256). */
typedef struct uocr_overlay uocr_overlay;
int uocr_overlay_check(const char *overlay_path, const char *source_path, size_t *matrix_count,
                       size_t *device_bytes);
int uocr_overlay_load(uocr_ctx *ctx, const char *overlay_path, const char *source_path,
                      uocr_overlay **out);
int uocr_overlay_get(const uocr_overlay *overlay, const char *name, const uocr_q8 **out);
size_t uocr_overlay_count(const uocr_overlay *overlay);
const char *uocr_overlay_name(const uocr_overlay *overlay, size_t index);
size_t uocr_overlay_device_bytes(const uocr_overlay *overlay);
int uocr_overlay_free(uocr_overlay *overlay);
int uocr_sha256_file(const char *path, char *hex_out);

#ifdef __cplusplus
}
#endif
#endif /* UOCR_Q8_H */
