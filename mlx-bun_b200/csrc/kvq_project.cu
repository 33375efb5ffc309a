// kvq_project.cu — the step before the append, fused: K/V projection of the
// layer input through MLX affine-quantized weights, the K and V RMSNorms,
// RoPE of K at the cache position, and the quantize-on-append into the
// cache rows the cache's state machine picks.  Replaces mlx-bun's
//   k = kProj(x); v = vProj(x) (or k, attention_k_eq_v);
//   k = rope(kNorm(k), offset); v = vNorm(v);
//   cache.updateAndFetchQuantized(k, v)
// (src/model/gemma4.ts:234-268; QuantizedLinear.forward,
// src/model/gemma4-base.ts:120-157; generated/gemma4-12b.ts:52-66), which
// runs as a quantized matmul per projection, two norms, a rope, two
// transposes and two quantize dispatches.
//
// Two launches, chained by programmatic dependent launch:
//   proj_partial_kernel: grid (splits, 2 * Hkv, row chunks), D threads.
//     CTA (s, (K|V, kv head h), a chunk of 1, 4 or 16 rows) accumulates,
//     for output column o = thread, sum_i x[r, i] * w[h*D + o, i] over its
//     contiguous run of weight groups, with w = scale * code + bias
//     dequantised in registers from the packed weight row (each weight byte
//     read once per row chunk) and the rows' inputs staged in shared memory
//     per group; f32 partials go to the workspace.  The split count spreads
//     a decode step's few rows over about two CTAs per SM; long chunks use
//     one split.
//   proj_epilogue_kernel: grid (rows, 2 * Hkv), D threads: the partials
//     summed in split order (deterministic) and rounded to the dtype (the
//     projection's output); RMSNorm (f32 mean of squares, x / sqrt(ms +
//     eps) rounded, times the weight, rounded); for K, RoPE on the first
//     `dims` elements (pairs (i, i + dims/2), or (2i, 2i + 1) traditional;
//     theta = scale * position * inv_freq, inv_freq = base^(-2i/dims) or
//     1 / freqs[i]; f32, rounded); then the affine quantize rule of
//     kvq_qrule.cuh per group, and the packed row, scales and biases
//     written at the destination row.  Optionally the dtype rows before
//     quantisation go to k_out / v_out (checking).
// Roofline: HBM on the weights (Hkv * D * hidden * wbits/8 per projection)
// for decode steps; the epilogue is a few microseconds of latency.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "kvq_attn_impl.cuh"
#include "kvq_qrule.cuh"

namespace kvq {
namespace proj {

using attn::dt_to_f;
using attn::f_to_dt;
using attn::round_dt;


struct W {
  const uint32_t* packed;
  const uint16_t* scales;
  const uint16_t* biases;  // nullable
  int bits, gs;
};

struct PP {
  const uint16_t* x;  // [R, hidden]
  W wk, wv;
  int v_from_k;
  int R, L, hidden, Hkv, D, ns;
  float* part;        // [2][Hkv][ns][R][D]
  // epilogue
  const uint16_t* k_norm;
  const uint16_t* v_norm;
  int norms;          // bit 0: K, bit 1: V
  float eps;
  int rope_dims, rope_trad;
  float rope_base, rope_scale;
  const float* rope_freqs;
  int64_t pos0;
  uint16_t* k_out;    // [B, Hkv, L, D] nullable
  uint16_t* v_out;
  // destination
  TripleView dk, dv;
  int64_t dst_row0;
  int bits, gs;       // cache quantisation
};

template <int WBITS, bool BF, int RC>
__global__ void __launch_bounds__(256) proj_partial_kernel(const PP p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ float xs[];  // [RC][gs]
  const int sel = blockIdx.y / p.Hkv, h = blockIdx.y - sel * p.Hkv;
  if (sel == 1 && p.v_from_k) return;
  const W w = sel ? p.wv : p.wk;
  const int tid = threadIdx.x, o = tid, D = p.D;
  const int r0 = blockIdx.z * RC, nr = min(RC, p.R - r0);
  const int G = p.hidden / w.gs;
  const int g0 = (int)((int64_t)blockIdx.x * G / p.ns), g1 = (int)((int64_t)(blockIdx.x + 1) * G / p.ns);
  constexpr int PER = 32 / WBITS;
  constexpr uint32_t MASK = (1u << WBITS) - 1u;
  const int gs = w.gs, wpg = gs / PER;          // packed words per group (a multiple of 4)
  const int64_t wrow = (int64_t)h * D + o;     // weight row of this output column
  const uint32_t* wp = w.packed + wrow * (p.hidden / PER);
  const uint16_t* sp = w.scales + wrow * G;
  const uint16_t* bp = w.biases ? w.biases + wrow * G : nullptr;
  float acc[RC];
#pragma unroll
  for (int r = 0; r < RC; r++) acc[r] = 0.0f;
  for (int g = g0; g < g1; g++) {
    __syncthreads();
    for (int idx = tid; idx < RC * gs; idx += blockDim.x) {
      const int r = idx / gs, j = idx - r * gs;
      xs[idx] = r < nr ? dt_to_f<BF>(p.x[(int64_t)(r0 + r) * p.hidden + (int64_t)g * gs + j]) : 0.0f;
    }
    __syncthreads();
    if (o >= D) continue;
    const float sc = dt_to_f<BF>(sp[g]), bi = bp ? dt_to_f<BF>(bp[g]) : 0.0f;
    const uint4* wv4 = reinterpret_cast<const uint4*>(wp + (int64_t)g * wpg);
    for (int q4 = 0; q4 < wpg / 4; q4++) {
      const uint4 u = __ldg(wv4 + q4);
      const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
#pragma unroll
        for (int e = 0; e < PER; e++) {
          const float wf = sc * (float)((q[k] >> (WBITS * e)) & MASK) + bi;
          const float* xr = xs + (q4 * 4 + k) * PER + e;
#pragma unroll
          for (int r = 0; r < RC; r++) acc[r] = fmaf(xr[r * gs], wf, acc[r]);
        }
      }
    }
  }
  if (o >= D) return;
  float* dst = p.part + ((((int64_t)sel * p.Hkv + h) * p.ns + blockIdx.x) * p.R + r0) * D + o;
#pragma unroll
  for (int r = 0; r < RC; r++)
    if (r < nr) dst[(int64_t)r * D] = acc[r];
}

// sum of v over the block (blockDim.x a multiple of 32, <= 256)
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

template <int BITS, bool BF>
__global__ void __launch_bounds__(256) proj_epilogue_kernel(const PP p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float row[256];
  __shared__ float red[8];
  const int r = blockIdx.x, sel = blockIdx.y / p.Hkv, h = blockIdx.y - sel * p.Hkv;
  const int o = threadIdx.x, D = p.D;
  const int b = r / p.L, l = r - b * p.L;
  const int src = (sel == 1 && p.v_from_k) ? 0 : sel;
  float x = 0.0f;
  if (o < D) {
    const float* part = p.part + (((int64_t)src * p.Hkv + h) * p.ns * p.R + r) * D + o;
    for (int s = 0; s < p.ns; s++) x += part[(int64_t)s * p.R * D];
    x = round_dt<BF>(x);  // the projection's output, in the dtype
  }
  if (p.norms & (1 << sel)) {
    // RMSNorm: x * (1 / sqrt(mean(x^2) + eps)) rounded, then * weight rounded
    const float ss = block_sum(o < D ? x * x : 0.0f, red);
    const float n = 1.0f / sqrtf(ss / (float)D + p.eps);
    const uint16_t* wn = sel ? p.v_norm : p.k_norm;
    if (o < D) {
      x = round_dt<BF>(x * n);
      if (wn) x = round_dt<BF>(x * dt_to_f<BF>(wn[o]));
    }
  }
  if (sel == 0 && p.rope_dims > 0) {
    __syncthreads();
    if (o < D) row[o] = x;
    __syncthreads();
    const int half = p.rope_dims / 2;
    if (o < 2 * half) {
      // pair index i, its two elements, and which of them this thread makes
      const int i = p.rope_trad ? o >> 1 : (o < half ? o : o - half);
      const int e1 = p.rope_trad ? 2 * i : i, e2 = p.rope_trad ? 2 * i + 1 : i + half;
      const bool first = o == e1;
      const float inv = p.rope_freqs ? 1.0f / p.rope_freqs[i]
                                     : exp2f(-((float)i / (float)half) * p.rope_base);
      const float theta = (p.rope_scale * (float)(p.pos0 + l)) * inv;
      const float cs = cosf(theta), sn = sinf(theta);
      const float x1 = row[e1], x2 = row[e2];
      x = round_dt<BF>(first ? x1 * cs - x2 * sn : x1 * sn + x2 * cs);
    }
  }
  uint16_t* dbg = sel ? p.v_out : p.k_out;
  if (dbg && o < D) dbg[(((int64_t)b * p.Hkv + h) * p.L + l) * D + o] = f_to_dt<BF>(x);
  __syncthreads();
  if (o < D) row[o] = x;
  __syncthreads();
  // quantize: thread t packs word t; the group's extremes are read from the row
  constexpr int PER = 32 / BITS;
  constexpr float NB = (float)((1 << BITS) - 1);
  const int words = D / PER, gs = p.gs, tpg = gs / PER;
  if (o >= words) return;
  const int g = o / tpg;
  float mn = row[g * gs], mx = mn;
  for (int j = 1; j < gs; j++) {
    mn = fminf(mn, row[g * gs + j]);
    mx = fmaxf(mx, row[g * gs + j]);
  }
  float scale, bias;
  quant_params(mn, mx, NB, scale, bias);
  uint32_t out = 0;
#pragma unroll
  for (int e = 0; e < PER; e++) out |= quant_code(row[o * PER + e], scale, bias, NB) << (BITS * e);
  const TripleView& dv = sel ? p.dv : p.dk;
  const int64_t drow = b * dv.batch_stride + h * dv.head_stride + p.dst_row0 + l;
  dv.packed[drow * words + o] = out;
  if (o % tpg == 0) {
    const int groups = D / gs;
    dv.scales[drow * groups + g] = f_to_dt<BF>(scale);
    dv.biases[drow * groups + g] = f_to_dt<BF>(bias);
  }
}

// rows per projection CTA: one decode row, a small batch, or 16-row chunks
inline int proj_rows(int R) { return R <= 1 ? 1 : R <= 4 ? 4 : 16; }

template <int WBITS, bool BF>
int32_t partial_for(int RC, dim3 grid, int threads, size_t smem, cudaStream_t st, const PP& p) {
  if (RC == 1) KVQ_CUDA_TRY(launch_pdl(proj_partial_kernel<WBITS, BF, 1>, grid, dim3(threads), smem, st, p));
  else if (RC == 4) KVQ_CUDA_TRY(launch_pdl(proj_partial_kernel<WBITS, BF, 4>, grid, dim3(threads), smem, st, p));
  else KVQ_CUDA_TRY(launch_pdl(proj_partial_kernel<WBITS, BF, 16>, grid, dim3(threads), smem, st, p));
  return KVQ_OK;
}

}  // namespace proj

using namespace proj;

size_t project_workspace_bytes(const ProjArgs& a, int Hkv, int D, int* splits) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int R = a.B * a.L;
  const int G = a.hidden / a.wk.gs;
  const int nrc = (R + proj_rows(R) - 1) / proj_rows(R);
  const int heads = a.v_from_k ? Hkv : 2 * Hkv;
  int ns = (2 * sms + heads * nrc - 1) / (heads * nrc);
  ns = std::max(1, std::min(ns, std::min(G, a.v_from_k ? G : a.hidden / a.wv.gs)));
  if (splits) *splits = ns;
  return attn::kPartialOff + (size_t)2 * Hkv * ns * R * D * sizeof(float);
}

int32_t launch_project_append(const ProjArgs& a, int Hkv, RowGeom g, int dtype, TripleView dk,
                              TripleView dv, int64_t dst_row0, void* ws, size_t ws_bytes,
                              cudaStream_t st) {
  const int D = g.D;
  int ns = 1;
  const size_t need = project_workspace_bytes(a, Hkv, D, &ns);
  int32_t rc = KVQ_OK;
  if (!ws) {
    int dev = 0;
    KVQ_CUDA_TRY(cudaGetDevice(&dev));
    ws = managed_workspace(dev, need, st, &rc);
    if (rc) return rc;
  } else if (ws_bytes < need) {
    return fail(KVQ_ERR_ARG, "workspace too small for the projection (" + std::to_string(need) + " bytes needed)");
  }
  PP p{};
  p.x = static_cast<const uint16_t*>(a.x);
  p.wk = W{a.wk.packed, static_cast<const uint16_t*>(a.wk.scales), static_cast<const uint16_t*>(a.wk.biases),
           a.wk.bits, a.wk.gs};
  p.wv = a.v_from_k ? p.wk
                    : W{a.wv.packed, static_cast<const uint16_t*>(a.wv.scales),
                        static_cast<const uint16_t*>(a.wv.biases), a.wv.bits, a.wv.gs};
  p.v_from_k = a.v_from_k ? 1 : 0;
  p.R = a.B * a.L;
  p.L = a.L;
  p.hidden = a.hidden;
  p.Hkv = Hkv;
  p.D = D;
  p.ns = ns;
  p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + attn::kPartialOff);
  p.k_norm = static_cast<const uint16_t*>(a.k_norm);
  p.v_norm = static_cast<const uint16_t*>(a.v_norm);
  p.norms = a.norms;
  p.eps = a.eps;
  p.rope_dims = a.rope_dims;
  p.rope_trad = a.rope_traditional ? 1 : 0;
  p.rope_base = a.rope_freqs ? 0.0f : (float)std::log2((double)a.rope_base);
  p.rope_scale = a.rope_scale;
  p.rope_freqs = a.rope_freqs;
  p.pos0 = a.pos0;
  p.k_out = static_cast<uint16_t*>(a.k_out);
  p.v_out = static_cast<uint16_t*>(a.v_out);
  p.dk = dk;
  p.dv = dv;
  p.dst_row0 = dst_row0;
  p.bits = g.bits;
  p.gs = g.gs;
  const bool bf = dtype == KVQ_DTYPE_BFLOAT16;
  const int threads = (D + 31) / 32 * 32;
  // projection: one V-less launch when V is K's projection
  const int RC = proj_rows(p.R);
  const dim3 g1(ns, 2 * Hkv, (p.R + RC - 1) / RC);
  const int wmax = std::max(a.wk.gs, a.v_from_k ? 0 : a.wv.gs);
  const size_t smem = (size_t)RC * wmax * sizeof(float);
  if (a.wk.bits != (a.v_from_k ? a.wk.bits : a.wv.bits))
    return fail(KVQ_ERR_ARG, "the K and V projections must share a bit width");
  rc = a.wk.bits == 4 ? (bf ? partial_for<4, true>(RC, g1, threads, smem, st, p)
                            : partial_for<4, false>(RC, g1, threads, smem, st, p))
                      : (bf ? partial_for<8, true>(RC, g1, threads, smem, st, p)
                            : partial_for<8, false>(RC, g1, threads, smem, st, p));
  if (rc) return rc;
  const dim3 g2(p.R, 2 * Hkv);
  auto ek = [&](auto kern) -> int32_t {
    KVQ_CUDA_TRY(launch_pdl(kern, g2, dim3(threads), 0, st, p));
    return KVQ_OK;
  };
  switch (g.bits * 2 + (bf ? 1 : 0)) {
    case 4 * 2: return ek(proj_epilogue_kernel<4, false>);
    case 4 * 2 + 1: return ek(proj_epilogue_kernel<4, true>);
    case 8 * 2: return ek(proj_epilogue_kernel<8, false>);
    default: return ek(proj_epilogue_kernel<8, true>);
  }
}

}  // namespace kvq
