// handles.h — the opaque handle types of include/uocr_q8.h (library-internal).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "kernels.h"

struct uocr_moe;

// One instantiated graph of the host-buffer decode call (copy in, decode
// kernel writing into pinned memory, status copy out), valid while the
// buffers it captured are the context's current ones.
struct HostDecodeGraph {
  const uocr_moe* layer = nullptr;
  uint64_t serial = 0;
  int mode = 0, outs = 0;
  const void* io = nullptr;
  const void* ws = nullptr;
  const void* pinned = nullptr;
  cudaGraphExec_t exec = nullptr;
};

struct uocr_ctx {
  int device = 0;
  int sms = 0;
  size_t scratch_limit = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  unsigned* status_dev = nullptr;
  unsigned* status_host = nullptr;  // pinned
  void* ws = nullptr;
  size_t ws_bytes = 0;
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
  void* io = nullptr;  // device staging of the *_host MoE entry point
  size_t io_bytes = 0;
  std::vector<HostDecodeGraph> host_graphs;  // at most kMaxHostGraphs, oldest replaced
  cudaStream_t capture_stream = nullptr;
  // a second stream, of the highest priority, for the critical chain of a call
  // that forks (the routing and the routed experts, while the shared expert
  // runs on `stream`), forked and joined through the two events
  cudaStream_t side_stream = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // uocr_ctx_set_wait_limit (0: the kernels' default) and the failure-detection
  // test hook uocr_ctx_hold_decode_barrier
  uint64_t wait_ns = 0;
  int hold_barrier = 0;
};

struct uocr_q8 {
  int device = 0;
  size_t rows = 0, cols = 0;
  int8_t* w = nullptr;
  float* s = nullptr;
  bool owns = false;
};

struct uocr_moe {
  int device = 0;
  uint64_t serial = 0;  // unique per created layer (graph cache key)
  size_t n_experts = 0, top_k = 0;
  int normalize = 0;
  float scale = 1.0f;
  int hidden = 0, width = 0, shared_width = 0;
  uocr::FfnView shared{};
  uocr::FfnView* experts_dev = nullptr;
  bool aligned = true;
  // Tensor-core prefill: TMA maps of every routed expert's weights and
  // scales, [3][n_experts] (gate, up, down); null when a shape does not
  // qualify.
  void* tc_maps = nullptr;
};

// Rotary table: (cos, sin) of every (position, pair), built on the host.
struct uocr_rope {
  int device = 0;
  int head_dim = 0, max_pos = 0;
  float theta = 0.0f;
  float2* table = nullptr;  // device [max_pos][head_dim/2]
};

// KV cache of `batch` sequences (LayerCache each): keys/values per (sequence,
// head) in the layout of uocr::KvLayout, device state {prefix, generated} per
// sequence; the host mirrors which sequences are prefilled.
struct uocr_kv {
  int device = 0;
  int batch = 0, heads = 0, head_dim = 0, width = 0, window = 0, max_prefix = 0;
  long long cap = 0;          // slots per sequence (max_prefix + window, rounded up when tiled)
  uocr::KvLayout layout{};
  float* keys = nullptr;
  float* values = nullptr;
  int* state = nullptr;
  std::vector<int> prefix;  // host mirror (0: not prefilled)
  bool tma = false;         // maps valid: the TMA attention kernel applies
  uocr::AttnMaps maps{};
  float* scores = nullptr;  // split attention scratch [batch][heads][cap] (tiled layout)
  int split = 0;            // attention form: 0 by batch size, 1 one CTA per head, 2 split
};
