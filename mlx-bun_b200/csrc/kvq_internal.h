// kvq_internal.h — shared declarations of libkvq's CUDA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "kvq.h"

namespace kvq {

// Thread-local error text behind kvq_last_error().
void set_error(const std::string& msg);
int32_t fail(int32_t code, const std::string& msg);
int32_t cuda_fail(cudaError_t e, const char* what);

#define KVQ_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return ::kvq::cuda_fail(_e, #expr); \
  } while (0)

// Geometry of one quantized row.
struct RowGeom {
  int D, bits, gs;
  int words() const { return D * bits / 32; }       // uint32 per packed row
  int groups() const { return D / gs; }              // scales (and biases) per row
};

// Base pointers + row strides of one triple (device side view).
struct TripleView {
  uint32_t* packed;
  uint16_t* scales;
  uint16_t* biases;
  int64_t batch_stride;  // rows
  int64_t head_stride;   // rows
};

// ---- quantize kernels (kvq_quant.cu) ----
// Quantize K and V rows of logical shape [B, H, S, D] (element strides
// (b, h, s), d stride 1) into rows dst_row0 + s of the two destination
// triples, in one launch.
int32_t launch_append_kv(const void* k, const int64_t* k_strides, const void* v,
                         const int64_t* v_strides, int B, int H, int S, RowGeom g, int dtype,
                         TripleView dk, TripleView dv, int64_t dst_row0, cudaStream_t st);
// Ragged: entry b writes its first counts[b] (nullable: S) rows at rows
// lens[b] + s (device arrays), then a second launch advances lens[b] by
// that count; entries that would pass `cap` rows are skipped and raise *err.
int32_t launch_append_ragged(const void* k, const int64_t* k_strides, const void* v,
                             const int64_t* v_strides, int B, int H, int S, RowGeom g, int dtype,
                             TripleView dk, TripleView dv, int64_t cap, int32_t* lens,
                             const int32_t* counts, int* err, cudaStream_t st);
// Contiguous rows -> contiguous triple.
int32_t launch_quantize_rows(const void* x, int64_t rows, RowGeom g, int dtype, uint32_t* packed,
                             uint16_t* scales, uint16_t* biases, cudaStream_t st);

// ---- fused projection + norms + RoPE + quantize-on-append (kvq_project.cu) ----
struct ProjWeights {
  const uint32_t* packed;  // [out, in * bits / 32]
  const void* scales;      // [out, in / gs], the activation dtype
  const void* biases;      // same shape, nullable
  int bits, gs;
};
struct ProjArgs {
  const void* x;  // [B, L, hidden] contiguous
  int B, L, hidden;
  ProjWeights wk, wv, wq;
  bool v_from_k;  // V is K's projection (before the norms)
  bool has_q;     // a query projection (Hq heads) into q_out
  int Hq;
  const void* k_norm;  // [D] nullable
  const void* v_norm;  // [D] nullable
  const void* q_norm;  // [D] nullable
  int norms;           // bit 0: RMSNorm on K, bit 1: on V, bit 2: on Q
  float eps;
  int rope_dims;       // 0: no RoPE
  bool rope_traditional;  // pairs (2i, 2i+1) instead of (i, i + dims/2)
  float rope_base, rope_scale;
  float rope_pre_scale;     // 0 or 1: none
  const float* rope_freqs;  // [rope_dims / 2] device, nullable
  int64_t pos0;        // position of row l = pos0 + l
  void* k_out;         // [B, Hkv, L, D] rows before quantisation, nullable
  void* v_out;
  void* q_out;         // [B, Hq, L, D] the query rows (with has_q)
};
// Workspace bytes of one launch (and the split count it uses).
size_t project_workspace_bytes(const ProjArgs& a, int Hkv, int D, int* splits);
int32_t launch_project_append(const ProjArgs& a, int Hkv, RowGeom g, int dtype, TripleView dk,
                              TripleView dv, int64_t dst_row0, void* ws, size_t ws_bytes,
                              cudaStream_t st);

// ---- attention (kvq_decode.cu / kvq_prefill.cu) ----
struct AttnArgs {
  TripleView k, v;
  int B, Hkv, Hq, N, D, bits, gs, dtype;
  float scale;
  const void* q;
  const int32_t* seq_lens;  // device, nullable
};

// Launch `kern` as a programmatic dependent of the previous kernel on the
// stream: it may be scheduled before that kernel finishes, so every kernel
// launched this way executes `griddepcontrol.wait` before its first access
// to global memory (and `griddepcontrol.launch_dependents` early, to let the
// next one do the same).  Hides the launch gap between the append, attention
// and merge kernels of a decode step.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

size_t decode_workspace_bytes(int B, int Hkv, int Hq, int N, int D);
// Exact workspace bytes one decode launch with these arguments uses, and the
// bytes at the start of the workspace that must be zero before it runs
// (error flag and split tickets).  With a budget, the launch is planned to
// fit in that many bytes where it can (see launch_decode's fit_to_ws).
int32_t decode_workspace_exact(const AttnArgs& a, size_t* bytes, size_t* zero_prefix,
                               size_t budget = SIZE_MAX);
// Fill AttnArgs from two views and a query (checks shapes; no CUDA calls).
int32_t make_attn_args(const kvq_qtensor* k, const kvq_qtensor* v, const void* q, int32_t q_heads,
                       float scale, const int32_t* seq_lens, AttnArgs& a);
// mode 0: normalized output in `out` (dtype); mode 1: partials (m, l, o).
// fit_to_ws: plan the launch to fit in ws_bytes (fewer CTAs) instead of
// refusing a workspace smaller than the full launch needs.
int32_t launch_decode(const AttnArgs& a, void* out, float* pm, float* pl, float* po, void* ws,
                      size_t ws_bytes, cudaStream_t st, bool fit_to_ws = false);
int32_t launch_merge(const float* m, const float* l, const float* o, int parts, int64_t pstride,
                     int rows, int D, int dtype, void* out, cudaStream_t st);
int32_t launch_prefill(const AttnArgs& a, int L, int mask_mode, int window, void* out, void* ws,
                       size_t ws_bytes, cudaStream_t st);
int32_t launch_debug_scores(const AttnArgs& a, int L, int mask_mode, int window, float* scores,
                            cudaStream_t st);

// Library-managed scratch per device (grown on demand, zero-filled; a
// buffer that a larger shape replaces stays allocated, since queued work or
// a captured graph may still use it).
void* managed_workspace(int device, size_t bytes, cudaStream_t st, int32_t* status);

// Every decode/prefill workspace starts with the device error flag (an int
// at offset 0) in a block of this many bytes.
constexpr size_t kWsFlagBytes = 256;

// Opt `kern` in to `smem` bytes of dynamic shared memory on device `dev`
// (the current device) and report its resident blocks per SM at `threads`
// threads.  The attribute is per device: done once per (kernel, device,
// shape) under a lock, then cached.
int32_t kernel_setup(const void* kern, int threads, int smem, int dev, int* blocks_per_sm);

// Device address of kvq_sdpa_decode_noalloc's scratch on `dev`, or nullptr
// while no call on that device has looked it up (kvq_noalloc.cu).
void* noalloc_scratch_if_known(int dev);

}  // namespace kvq
