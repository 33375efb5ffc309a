// kvq_project.cu — the step before the append, fused: K/V (and Q)
// projection of the layer input through MLX affine-quantized weights, the
// K, V (and Q) RMSNorms, RoPE of K (and Q) at the cache position, the
// quantize-on-append of K and V into the cache rows the cache's state
// machine picks, and the query rows into the caller's buffer.  Replaces
// mlx-bun's
//   q = qNorm(qProj(x)); k = kProj(x); v = vProj(x) (or k, attention_k_eq_v);
//   k = rope(kNorm(k), offset); v = vNorm(v);
//   cache.updateAndFetchQuantized(k, v); q = rope(transpose(q), offset)
// (src/model/gemma4.ts:224-268; QuantizedLinear.forward,
// src/model/gemma4-base.ts:120-157; generated/gemma4-12b.ts:52-74), which
// runs as a quantized matmul per projection, three norms, two ropes, three
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

#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "kvq_attn_impl.cuh"
#include "kvq_qrule.cuh"

namespace kvq {
namespace proj {

using attn::dt_to_f;
using attn::f_to_dt;
using attn::round_dt;
using attn::pack_h2;


struct W {
  const uint32_t* packed;
  const uint16_t* scales;
  const uint16_t* biases;  // nullable
  int bits, gs;
};

// Projections and heads.  A compute unit is one head of one projection —
// the K heads, then the V heads (none when V is K's projection), then the
// Q heads (none without a query projection) — and owns D output rows.  A
// finish unit is one head's row after the projection: the K heads, the V
// heads (finished from K's rows when V is K's projection), the Q heads.
struct PP {
  const uint16_t* x;  // [R, hidden]
  W wk, wv, wq;
  int v_from_k;
  int R, L, hidden, Hkv, D, ns;
  int Hq, nv, nq;     // query heads; V and Q compute units (0 or Hkv, 0 or Hq)
  float* part;        // [compute unit][ns][R][D]
  // epilogue
  const uint16_t* k_norm;
  const uint16_t* v_norm;
  const uint16_t* q_norm;
  int norms;          // bit 0: K, bit 1: V, bit 2: Q
  float eps;
  int rope_dims, rope_trad;
  float rope_base, rope_scale, rope_pre;
  const float* rope_freqs;
  int64_t pos0;
  uint16_t* k_out;    // [B, Hkv, L, D] nullable
  uint16_t* v_out;
  uint16_t* q_out;    // [B, Hq, L, D] (with a query projection)
  // destination
  TripleView dk, dv;
  int64_t dst_row0;
  int bits, gs;       // cache quantisation
  int nb2;            // cluster path: weight loads per thread staged in shared memory
};

__device__ __forceinline__ int units_of(const PP& p) { return p.Hkv + p.nv + p.nq; }

// compute unit u -> projection (0 K, 1 V, 2 Q) and head
__device__ __forceinline__ void unit_of(const PP& p, int u, int& sel, int& h) {
  if (u < p.Hkv) {
    sel = 0;
    h = u;
  } else if (u < p.Hkv + p.nv) {
    sel = 1;
    h = u - p.Hkv;
  } else {
    sel = 2;
    h = u - p.Hkv - p.nv;
  }
}

__device__ __forceinline__ const W& w_of(const PP& p, int sel) {
  return sel == 0 ? p.wk : sel == 1 ? p.wv : p.wq;
}

// finish unit f -> projection, head and the compute unit holding its rows
__device__ __forceinline__ void finish_of(const PP& p, int f, int& sel, int& h, int& src) {
  if (f < p.Hkv) {
    sel = 0;
    h = f;
    src = f;
  } else if (f < 2 * p.Hkv) {
    sel = 1;
    h = f - p.Hkv;
    src = p.nv ? p.Hkv + h : h;
  } else {
    sel = 2;
    h = f - 2 * p.Hkv;
    src = p.Hkv + p.nv + h;
  }
}

template <int WBITS, bool BF, int RC>
__global__ void __launch_bounds__(256) proj_partial_kernel(const PP p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ float xs[];  // [RC][gs]
  int sel, h;
  unit_of(p, blockIdx.y, sel, h);
  const W w = w_of(p, sel);
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
  float* dst = p.part + (((int64_t)blockIdx.y * p.ns + blockIdx.x) * p.R + r0) * D + o;
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

// What finish_row needs besides the projected value, fetched / computed
// ahead of it (none of it depends on the projection): thread o's norm
// weight and, for K rows, the cosine and sine of its RoPE pair at the row's
// position.
struct RowConsts {
  float wn;      // norm weight (1 without one)
  float cs, sn;  // RoPE rotation (K, o < rope_dims)
};

template <bool BF>
__device__ __forceinline__ RowConsts row_consts(const PP& p, int sel, int r) {
  const int o = threadIdx.x;
  RowConsts c{1.0f, 1.0f, 0.0f};
  if (o >= p.D) return c;
  const uint16_t* wn = sel == 0 ? p.k_norm : sel == 1 ? p.v_norm : p.q_norm;
  if ((p.norms & (1 << sel)) && wn) c.wn = dt_to_f<BF>(wn[o]);
  const int half = p.rope_dims / 2;
  if (sel != 1 && o < 2 * half) {
    const int l = r % p.L;
    const int i = p.rope_trad ? o >> 1 : (o < half ? o : o - half);
    const float inv = p.rope_freqs ? 1.0f / p.rope_freqs[i]
                                   : exp2f(-((float)i / (float)half) * p.rope_base);
    const float theta = (p.rope_scale * (float)(p.pos0 + l)) * inv;
    c.cs = cosf(theta);
    c.sn = sinf(theta);
  }
  return c;
}

// Everything after the projection for one output row (token r) of head h:
// `x` is thread o's projected value (the dtype-rounded sum), sel 0 / 1 / 2
// = K / V / Q.  RMSNorm, RoPE (K and Q), then for Q the row into q_out, for
// K and V the checking copy and the quantize-on-append.
// Called by the whole CTA (it synchronises); `row` holds D floats, `red` 32.
template <int BITS, bool BF>
__device__ void finish_row(const PP& p, int sel, int h, int r, float x, const RowConsts& rc,
                           float* row, float* red) {
  const int o = threadIdx.x, D = p.D;
  const int b = r / p.L, l = r - b * p.L;
  if (p.norms & (1 << sel)) {
    // RMSNorm: x * (1 / sqrt(mean(x^2) + eps)) rounded, then * weight rounded
    const float ss = block_sum(o < D ? x * x : 0.0f, red);
    const float n = 1.0f / sqrtf(ss / (float)D + p.eps);
    const uint16_t* wn = sel == 0 ? p.k_norm : sel == 1 ? p.v_norm : p.q_norm;
    if (o < D) {
      x = round_dt<BF>(x * n);
      if (wn) x = round_dt<BF>(x * rc.wn);
    }
  }
  if (sel != 1 && p.rope_dims > 0) {
    // the pre-rope input scale (a weak scalar: rounded to the dtype first)
    if (p.rope_pre != 0.0f && o < p.rope_dims) x = round_dt<BF>(x * round_dt<BF>(p.rope_pre));
    __syncthreads();
    if (o < D) row[o] = x;
    __syncthreads();
    const int half = p.rope_dims / 2;
    if (o < 2 * half) {
      // the pair's two elements, and which of them this thread makes
      const int i = p.rope_trad ? o >> 1 : (o < half ? o : o - half);
      const int e1 = p.rope_trad ? 2 * i : i, e2 = p.rope_trad ? 2 * i + 1 : i + half;
      const float x1 = row[e1], x2 = row[e2];
      x = round_dt<BF>(o == e1 ? x1 * rc.cs - x2 * rc.sn : x1 * rc.sn + x2 * rc.cs);
    }
  }
  if (sel == 2) {  // the query row, in the layout attention reads
    if (o < D) p.q_out[(((int64_t)b * p.Hq + h) * p.L + l) * D + o] = f_to_dt<BF>(x);
    return;
  }
  uint16_t* dbg = sel ? p.v_out : p.k_out;
  if (dbg && o < D) dbg[(((int64_t)b * p.Hkv + h) * p.L + l) * D + o] = f_to_dt<BF>(x);
  // quantize: the group's extremes by warp shuffles (a group is gs / 32
  // whole warps; D is a multiple of 32, so warps are wholly in or out of
  // the row), then each thread's code, OR-ed into its word across the
  // word's lanes
  constexpr int PER = 32 / BITS;
  constexpr float NB = (float)((1 << BITS) - 1);
  const int gs = p.gs, warp = threadIdx.x >> 5;
  float mn = x, mx = x;
  if (o < D) {
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
  }
  __syncthreads();  // `red` may still be read by the norm's block sum
  if (o < D && (threadIdx.x & 31) == 0) {
    red[warp] = mn;
    red[16 + warp] = mx;
  }
  __syncthreads();
  if (o >= D) return;
  const int wpg = gs / 32, w0 = (o / gs) * wpg;
  mn = red[w0];
  mx = red[16 + w0];
  for (int k = 1; k < wpg; k++) {
    mn = fminf(mn, red[w0 + k]);
    mx = fmaxf(mx, red[16 + w0 + k]);
  }
  float scale, bias;
  quant_params(mn, mx, NB, scale, bias);
  uint32_t word = quant_code(x, scale, bias, NB) << (BITS * (o % PER));
#pragma unroll
  for (int off = 1; off < PER; off <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, off);
  const TripleView& dv = sel ? p.dv : p.dk;
  const int64_t drow = b * dv.batch_stride + h * dv.head_stride + p.dst_row0 + l;
  if (o % PER == 0) dv.packed[drow * (D / PER) + o / PER] = word;
  if (o % gs == 0) {
    const int groups = D / gs, g = o / gs;
    dv.scales[drow * groups + g] = f_to_dt<BF>(scale);
    dv.biases[drow * groups + g] = f_to_dt<BF>(bias);
  }
}

template <int BITS, bool BF>
__global__ void __launch_bounds__(256) proj_epilogue_kernel(const PP p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float row[256];
  __shared__ float red[32];
  const int r = blockIdx.x;
  int sel, h, src;
  finish_of(p, blockIdx.y, sel, h, src);
  const int o = threadIdx.x, D = p.D;
  float x = 0.0f;
  if (o < D) {
    // the split partials, loaded together, summed in split order
    const float* part = p.part + ((int64_t)src * p.ns * p.R + r) * D + o;
    const int64_t ss = (int64_t)p.R * D;
    for (int s0 = 0; s0 < p.ns; s0 += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; k++) v[k] = s0 + k < p.ns ? part[(s0 + k) * ss] : 0.0f;
#pragma unroll
      for (int k = 0; k < 8; k++) x += v[k];
    }
    x = round_dt<BF>(x);  // the projection's output, in the dtype
  }
  finish_row<BITS, BF>(p, sel, h, r, x, row_consts<BF>(p, sel, r), row, red);
}

// The same per-row work with one warp per row (prefill: many rows).  One
// CTA per token, one warp per finish unit (a K, V or Q head): the CTA first computes the
// token's RoPE rotations (cos, sin of each pair's angle) once into shared
// memory — they are the same for every kv head — then each warp works on
// its row with no block barrier.  Lane l holds elements l + 32 k (k < E =
// D / 32): the norm's sum of squares and each group's min / max are warp
// shuffles (a group is gs / 32 of the lane's elements), RoPE reads the
// pair partner from the warp's row in shared memory, and a packed word's
// lanes OR their codes together by shuffles.
template <int BITS, bool BF, int E>
__global__ void __launch_bounds__(1024) proj_epilogue_warp_kernel(const PP p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ float esm[];  // cos [D/2], sin [D/2], then one row of D per warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x;
  int sel, h, src;
  finish_of(p, warp, sel, h, src);
  const int D = p.D;
  const int b = r / p.L, l = r - b * p.L;
  float* rcos = esm;
  float* rsin = esm + D / 2;
  // the token's rotations (inputs only: computed before the dependency wait)
  const int half = p.rope_dims / 2;
  if (p.rope_dims > 0) {
    const float pos = p.rope_scale * (float)(p.pos0 + l);
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float inv = p.rope_freqs ? 1.0f / p.rope_freqs[i]
                                     : exp2f(-((float)i / (float)half) * p.rope_base);
      float sn, cs;
      sincosf(pos * inv, &sn, &cs);
      rcos[i] = cs;
      rsin[i] = sn;
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  float* row = esm + D + warp * D;
  float x[E];
  const float* part = p.part + ((int64_t)src * p.ns * p.R + r) * D;
#pragma unroll
  for (int k = 0; k < E; k++) x[k] = 0.0f;
  for (int s2 = 0; s2 < p.ns; s2++) {  // every element's load of a split in flight together
    float v[E];
#pragma unroll
    for (int k = 0; k < E; k++) v[k] = part[(int64_t)s2 * p.R * D + lane + 32 * k];
#pragma unroll
    for (int k = 0; k < E; k++) x[k] += v[k];
  }
#pragma unroll
  for (int k = 0; k < E; k++) x[k] = round_dt<BF>(x[k]);  // the projection's output, in the dtype
  if (p.norms & (1 << sel)) {
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < E; k++) ss += x[k] * x[k];
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float n = 1.0f / sqrtf(ss / (float)D + p.eps);
    const uint16_t* wn = sel == 0 ? p.k_norm : sel == 1 ? p.v_norm : p.q_norm;
#pragma unroll
    for (int k = 0; k < E; k++) {
      x[k] = round_dt<BF>(x[k] * n);
      if (wn) x[k] = round_dt<BF>(x[k] * dt_to_f<BF>(wn[lane + 32 * k]));
    }
  }
  if (sel != 1 && p.rope_dims > 0) {
#pragma unroll
    for (int k = 0; k < E; k++) {
      const int e = lane + 32 * k;
      if (p.rope_pre != 0.0f && e < p.rope_dims) x[k] = round_dt<BF>(x[k] * round_dt<BF>(p.rope_pre));
      row[e] = x[k];
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < E; k++) {
      const int e = lane + 32 * k;
      if (e < 2 * half) {
        const int i = p.rope_trad ? e >> 1 : (e < half ? e : e - half);
        const int e1 = p.rope_trad ? 2 * i : i, e2 = p.rope_trad ? 2 * i + 1 : i + half;
        const float cs = rcos[i], sn = rsin[i];
        const float x1 = row[e1], x2 = row[e2];
        x[k] = round_dt<BF>(e == e1 ? x1 * cs - x2 * sn : x1 * sn + x2 * cs);
      }
    }
  }
  if (sel == 2) {  // the query row, in the layout attention reads
    uint16_t* qrow = p.q_out + (((int64_t)b * p.Hq + h) * p.L + l) * D;
#pragma unroll
    for (int k = 0; k < E; k++) qrow[lane + 32 * k] = f_to_dt<BF>(x[k]);
    return;
  }
  uint16_t* dbg = sel ? p.v_out : p.k_out;
  if (dbg) {
    uint16_t* drow = dbg + (((int64_t)b * p.Hkv + h) * p.L + l) * D;
#pragma unroll
    for (int k = 0; k < E; k++) drow[lane + 32 * k] = f_to_dt<BF>(x[k]);
  }
  // quantize: group j = lane elements k in [j * kpg, (j + 1) * kpg)
  constexpr int PER = 32 / BITS;
  constexpr float NB = (float)((1 << BITS) - 1);
  const int gs = p.gs, kpg = gs / 32, groups = D / gs;
  const TripleView& dv = sel ? p.dv : p.dk;
  const int64_t drow = b * dv.batch_stride + h * dv.head_stride + p.dst_row0 + l;
#pragma unroll
  for (int k0 = 0; k0 < E; k0 += 1) {
    if (k0 % kpg) continue;
    float mn = x[k0], mx = x[k0];
#pragma unroll
    for (int k = 1; k < 4; k++)
      if (k < kpg && k0 + k < E) {
        mn = fminf(mn, x[k0 + k]);
        mx = fmaxf(mx, x[k0 + k]);
      }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    float scale, bias;
    quant_params(mn, mx, NB, scale, bias);
    const int grp = k0 / kpg;
    if (lane == 0) {
      dv.scales[drow * groups + grp] = f_to_dt<BF>(scale);
      dv.biases[drow * groups + grp] = f_to_dt<BF>(bias);
    }
#pragma unroll
    for (int k = 0; k < 4; k++)
      if (k < kpg && k0 + k < E) {
        uint32_t word = quant_code(x[k0 + k], scale, bias, NB) << (BITS * (lane % PER));
#pragma unroll
        for (int off = 1; off < PER; off <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, off);
        if (lane % PER == 0) dv.packed[drow * (D / PER) + (lane + 32 * (k0 + k)) / PER] = word;
      }
  }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool full) {
  const uint32_t d = attn::smem_u32(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
               "r"(full ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Decode-sized steps (R <= 4 rows): one launch.  A cluster of CS CTAs per
// (K|V, kv head, row chunk) splits the hidden dimension; thread o owns
// output column o.  Each thread first issues everything it will read —
// its weight-row slice (16-byte loads: the first kNB into registers, up to
// nb2 more by cp.async into shared memory), its group scales and biases, the
// norm weight and the RoPE table before the dependency wait, its share of
// the input slice after it — then stages the inputs in shared memory and
// accumulates per group
//   s * sum(code * x) + b * sum(x)
// (the affine dequantisation factored out of the dot product; codes turned
// into floats by one byte permute each, see code_hi / code_lo; four independent
// partial sums).  The cluster's CTA 0 sums the CS partials from the
// others' shared memory in rank order (deterministic) and runs finish_row.
// With V = K's projection, the K cluster finishes both.  256 threads of at
// most 128 registers: two CTAs fit an SM, so the next step's CTAs are
// resident (waiting on the dependency) before this step ends.
constexpr int kMaxG = 8;    // weight groups per CTA
constexpr int kNB = 8;      // 16-byte weight loads per thread issued up front
constexpr int kNB2 = 8;     // further ones staged in shared memory (up to 32 KB per CTA)

// Codes as floats by one byte permute each (byte K of `w` into the float's
// bits, exponent byte 0x4B above it):
//  * 4-bit: the word's nibbles pre-shifted to bits 3..6 of their bytes
//    (code_hi) land in mantissa bits 19..22: 2^19 (16 + c).  Then
//      sum(x * 2^19 (16 + c)) * 2^-19 - 16 * sum(x) = sum(x * c),
//    exact products (fp16 / bf16 x), about 1.5 bits of the f32 sum lost to
//    the offset — far below the dtype's precision;
//  * 8-bit: the code lands in the low mantissa byte: 2^23 + c, and one
//    subtraction gives c exactly (code_lo).
template <int K>
__device__ __forceinline__ float code_hi(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4Bu, 0x4055u | (K << 8)));
}
template <int K>
__device__ __forceinline__ float code_lo(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u | K)) - 8388608.0f;
}

template <int WBITS, int BITS, bool BF, int RC, int CS>
__global__ void __launch_bounds__(256, 2) proj_cluster_kernel(const PP p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float row[256];
  __shared__ float red[32];
  extern __shared__ __align__(16) float sm[];  // wsm[nb2][D], part[RC][D], sumx[RC][kMaxG], xs[RC][span]
  const int rank = (int)cluster.block_rank();
  int sel, h;
  unit_of(p, blockIdx.y, sel, h);
  const W w = w_of(p, sel);
  const int o = threadIdx.x, D = p.D;
  const int G = p.hidden / w.gs, gs = w.gs;
  const int g0 = rank * G / CS, g1 = (rank + 1) * G / CS, ng = g1 - g0;
  const int span = ng * gs;
  uint4* wsm = reinterpret_cast<uint4*>(sm);
  float* part = sm + p.nb2 * D * 4;
  float* sumx = part + RC * D;
  float* xs = sumx + RC * kMaxG;
  const int r0 = blockIdx.z * RC, nr = min(RC, p.R - r0);
  constexpr int PER = 32 / WBITS;
  constexpr int E4 = 4 * PER;            // elements per 16-byte load
  const int u4pg = gs / E4;              // 16-byte loads per group: 1, 2, 4 or 8
  const int lg = __ffs(u4pg) - 1;        // log2(u4pg)
  const int n4 = ng * u4pg;
  const int64_t wrow = (int64_t)h * D + o;
  const uint4* wp = reinterpret_cast<const uint4*>(w.packed + wrow * (p.hidden / PER)) +
                    (int64_t)g0 * u4pg;
  // 1. the layer's parameters — weights, scales / biases (raw), norm weight,
  //    RoPE table — are loaded before waiting for the preceding kernel (they
  //    are not its output: the entry point requires it), so they stream in
  //    while that kernel finishes; the input rows only after the wait
  uint4 q[kNB];
#pragma unroll
  for (int j = 0; j < kNB; j++) q[j] = j < n4 ? __ldg(wp + j) : make_uint4(0, 0, 0, 0);
  const int nb2 = max(0, min(n4 - kNB, p.nb2));
#pragma unroll
  for (int j = 0; j < kNB2; j++)
    if (j < nb2) cp_async16(wsm + j * D + o, wp + kNB + j, true);
  cp_async_commit();
  // (scale | bias << 16) of the slice's groups, in order: each group's fold
  // takes sb[0] and shifts the rest down, so no index is computed
  uint32_t sb[kMaxG];
  const uint16_t* sp = w.scales + wrow * G + g0;
  const uint16_t* bp = w.biases ? w.biases + wrow * G + g0 : nullptr;
#pragma unroll
  for (int k = 0; k < kMaxG; k++) {
    const uint32_t s16 = k < ng ? __ldg(sp + k) : (uint16_t)0;
    const uint32_t b16 = (k < ng && bp) ? __ldg(bp + k) : (uint16_t)0;
    sb[k] = s16 | (b16 << 16);
  }
  RowConsts rcs[RC], rcv[RC];
  if (rank == 0) {
#pragma unroll
    for (int r = 0; r < RC; r++) {
      rcs[r] = row_consts<BF>(p, sel, r0 + r < p.R ? r0 + r : 0);
      rcv[r] = (p.v_from_k && sel == 0) ? row_consts<BF>(p, 1, r0 + r < p.R ? r0 + r : 0) : rcs[r];
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int kXL = RC == 1 ? 4 : 2;  // input elements per thread and row held in flight
  uint16_t xv[RC][kXL];
#pragma unroll
  for (int r = 0; r < RC; r++)
#pragma unroll
    for (int t = 0; t < kXL; t++) {
      const int j = o + t * D;
      xv[r][t] = (r < nr && j < span) ? __ldg(p.x + (int64_t)(r0 + r) * p.hidden + (int64_t)g0 * gs + j)
                                      : (uint16_t)0;
    }
  // 2. the input slice into shared memory (slices longer than kXL * D
  //    elements per row take the rest with plain loads)
#pragma unroll
  for (int r = 0; r < RC; r++) {
#pragma unroll
    for (int t = 0; t < kXL; t++) {
      const int j = o + t * D;
      if (j < span) xs[r * span + j] = dt_to_f<BF>(xv[r][t]);
    }
    for (int j = o + kXL * D; j < span; j += D)
      xs[r * span + j] = r < nr ? dt_to_f<BF>(p.x[(int64_t)(r0 + r) * p.hidden + (int64_t)g0 * gs + j])
                                : 0.0f;
  }
  __syncthreads();
  // sum(x) per (row, group) of the slice: one warp per pair
  {
    const int warp = o >> 5, lane = o & 31, nw = blockDim.x >> 5;
    for (int pr = warp; pr < RC * ng; pr += nw) {
      const int r = pr / ng, gl = pr - r * ng;
      float t = 0.0f;
      for (int j = lane; j < gs; j += 32) t += xs[r * span + gl * gs + j];
#pragma unroll
      for (int off = 16; off; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      if (lane == 0) sumx[r * kMaxG + gl] = t;
    }
  }
  __syncthreads();
  // 3. the dot products, group by group
  float out[RC], a[RC][4];
#pragma unroll
  for (int r = 0; r < RC; r++) out[r] = a[r][0] = a[r][1] = a[r][2] = a[r][3] = 0.0f;
  auto consume = [&](const uint4& v4, int j) {
    const uint32_t qq[4] = {v4.x, v4.y, v4.z, v4.w};
    const float* xb = xs + j * E4;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      // the word's codes one per byte: 4-bit words split into even / odd
      // elements at bits 3..6 of each byte; 8-bit words are bytes already
      float cf[PER];
      if (WBITS == 4) {
        const uint32_t b0 = (qq[kk] << 3) & 0x78787878u;
        const uint32_t b1 = (qq[kk] >> 1) & 0x78787878u;
        cf[0] = code_hi<0>(b0); cf[1] = code_hi<0>(b1);
        cf[2] = code_hi<1>(b0); cf[3] = code_hi<1>(b1);
        cf[4] = code_hi<2>(b0); cf[5] = code_hi<2>(b1);
        cf[6] = code_hi<3>(b0); cf[7] = code_hi<3>(b1);
      } else {
        cf[0] = code_lo<0>(qq[kk]); cf[1] = code_lo<1>(qq[kk]);
        cf[2] = code_lo<2>(qq[kk]); cf[3] = code_lo<3>(qq[kk]);
      }
#pragma unroll
      for (int r = 0; r < RC; r++) {
#pragma unroll
        for (int e4 = 0; e4 < PER; e4 += 4) {
          const float4 xv4 = *reinterpret_cast<const float4*>(xb + r * span + kk * PER + e4);
          a[r][0] = fmaf(xv4.x, cf[e4], a[r][0]);
          a[r][1] = fmaf(xv4.y, cf[e4 + 1], a[r][1]);
          a[r][2] = fmaf(xv4.z, cf[e4 + 2], a[r][2]);
          a[r][3] = fmaf(xv4.w, cf[e4 + 3], a[r][3]);
        }
      }
    }
    if (((j + 1) & (u4pg - 1)) == 0) {  // the group's last load (u4pg: a power of two)
      const int k = j >> lg;
      const uint32_t v = sb[0];
#pragma unroll
      for (int t = 0; t + 1 < kMaxG; t++) sb[t] = sb[t + 1];
      const float s = dt_to_f<BF>((uint16_t)(v & 0xffffu)), b = dt_to_f<BF>((uint16_t)(v >> 16));
#pragma unroll
      for (int r = 0; r < RC; r++) {
        const float sx = sumx[r * kMaxG + k];
        const float acc = (a[r][0] + a[r][1]) + (a[r][2] + a[r][3]);
        const float dot = WBITS == 4 ? fmaf(acc, 1.0f / 524288.0f, -16.0f * sx)  // sum(x * code)
                                     : acc;
        out[r] = fmaf(s, dot, fmaf(b, sx, out[r]));
        a[r][0] = a[r][1] = a[r][2] = a[r][3] = 0.0f;
      }
    }
  };
#pragma unroll
  for (int j = 0; j < kNB; j++) {
    if (j >= n4) break;
    consume(q[j], j);
  }
  cp_async_wait<0>();  // this thread's own copies: visible to it past the wait
  for (int j = 0; j < nb2; j++) consume(wsm[j * D + o], kNB + j);
  for (int j = kNB + nb2; j < n4; j++) consume(__ldg(wp + j), j);
#pragma unroll
  for (int r = 0; r < RC; r++) part[r * D + o] = out[r];
  cluster.sync();
  float xsum[RC];
#pragma unroll
  for (int r = 0; r < RC; r++) xsum[r] = 0.0f;
  if (rank == 0) {
#pragma unroll
    for (int r = 0; r < RC; r++) {
      float v[CS];
#pragma unroll
      for (int c = 0; c < CS; c++) v[c] = cluster.map_shared_rank(part, c)[r * D + o];
      float t = 0.0f;
#pragma unroll
      for (int c = 0; c < CS; c++) t += v[c];
      xsum[r] = round_dt<BF>(t);  // the projection's output, in the dtype
    }
  }
  cluster.sync();  // the other CTAs' shared memory stays alive until read
  if (rank != 0) return;
#pragma unroll
  for (int r = 0; r < RC; r++) {
    if (r >= nr) break;
    finish_row<BITS, BF>(p, sel, h, r0 + r, xsum[r], rcs[r], row, red);
    if (p.v_from_k && sel == 0) finish_row<BITS, BF>(p, 1, h, r0 + r, xsum[r], rcv[r], row, red);
  }
}

// Prefill-sized steps (more than 4 token rows): the projection on tensor
// cores, mma.sync m16n8k16 with f32 accumulation, then proj_epilogue_kernel.
// The GEMM is W x^T: M = the output features of K (and V) — all kv heads'
// rows, 128 per CTA — N = the token rows, 64 per CTA, K = hidden.  As in
// the decode attention's Q K^T, the codes enter the MMA exactly: a pair of
// codes as fp16 subnormals (units of 2^-24; one shift and mask per
// register for 4-bit, one byte permute for 8-bit), x as fp16 (exact: bf16
// inputs are first scaled per (group, token) block by a power of two into
// fp16's range, and the factor comes back at the fold), and per weight
// group
//   out += (s * 2^24) * sum(code * x 2^-24) + b * sum(x)
// between k-steps.  The k order inside a 16-element k-step is permuted so
// that each A register comes from one packed word: 4-bit lane t takes the
// nibble pair (t, t+4) of the step's two words; 8-bit lane t takes word t
// (its bytes (0, 1) and (2, 3)).  proj_xprep_kernel writes x once in that
// order as fp16, [group][k-step][token][16 halves], with sum(x) per
// (group, token); the GEMM then streams weights and inputs group by group
// through a kStages-deep cp.async ring (16-byte copies, zero-filled past
// the last row / token), so each lane reads its B fragment with one 8-byte
// shared load and its A words with one (4-bit) or two (8-bit).
constexpr int kMT = 128;    // output rows per CTA
constexpr int kNT = 64;     // token rows per CTA
constexpr int kStages = 4;  // cp.async ring depth, in weight groups

struct MmaGeo {
  int gs, wbits;
  __host__ __device__ constexpr MmaGeo(int g, int w) : gs(g), wbits(w) {}
  __host__ __device__ constexpr int row_bytes() const { return gs * wbits / 8; }   // codes of a row's group
  __host__ __device__ constexpr int row_pitch() const { return row_bytes() + 16; }  // padded: no bank conflicts
  __host__ __device__ constexpr int ksteps() const { return gs / 16; }
  __host__ __device__ constexpr int w_bytes() const { return kMT * row_pitch(); }
  __host__ __device__ constexpr int x_bytes() const { return ksteps() * kNT * 32; }
  __host__ __device__ constexpr int stage_bytes() const { return w_bytes() + x_bytes() + 2 * kNT * 4 + 2 * kMT * 4; }
};

// x [R, hidden] (dtype) -> xp [G][ksteps][R][16 halves] fp16 in the MMA's k
// order, and xsum [G][R] = sum(x) of each group.  Thread: 8 consecutive
// elements of one token (one 16-byte load).
template <int WBITS, bool BF>
__global__ void __launch_bounds__(256) proj_xprep_kernel(const PP p, uint8_t* xp, float* xsum,
                                                         float* xfac) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int gs = p.wk.gs, G = p.hidden / gs, cpg = gs / 8;  // 16-byte chunks per group
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)p.R * (p.hidden / 8);
  const bool live = i < total;
  const int64_t ii = live ? i : 0;
  const int n = (int)(ii / (p.hidden / 8)), ch = (int)(ii - (int64_t)n * (p.hidden / 8));
  const int grp = ch / cpg, c = ch - grp * cpg;
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p.x + (int64_t)n * p.hidden) + ch);
  const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
  float v[8], part = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    v[j] = dt_to_f<BF>((uint16_t)((j & 1) ? (wv[j / 2] >> 16) : (wv[j / 2] & 0xffffu)));
    part += v[j];
  }
  // the cpg lanes of one (token, group) are consecutive and aligned
  for (int off = 1; off < cpg; off <<= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  // bf16 inputs: the block's values times a power of two 2^-e that brings
  // its largest magnitude into [2^14, 2^15) — exact, inside fp16's range
  // whatever the bf16 exponents; the GEMM multiplies the block's dot
  // products by 2^e again
  float fac = 1.0f;
  if (BF) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
    for (int off = 1; off < cpg; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (amax > 0.0f) {
      int e = ((__float_as_uint(amax) >> 23) & 0xff) - 127 - 14;  // amax in [2^(e+14), 2^(e+15))
      e = max(-126, min(126, e));
      fac = __uint_as_float((uint32_t)(127 + e) << 23);
      const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] *= inv;
    }
  }
  if (!live) return;
  const int64_t xi = (int64_t)grp * ((p.R + 3) & ~3) + n;
  if (c == 0) {
    xsum[xi] = part;
    if (BF) xfac[xi] = fac;
  }
  const int s16 = c / 2, which = c & 1;  // k-step, first / second 8 elements of it
  uint8_t* dst = xp + (((int64_t)grp * (gs / 16) + s16) * p.R + n) * 32;
  if (WBITS == 4) {
    // lane t's halves: (x[t], x[t+4]) of the step's word `which`
#pragma unroll
    for (int tt = 0; tt < 4; tt++)
      *reinterpret_cast<uint32_t*>(dst + tt * 8 + which * 4) = pack_h2(v[tt], v[tt + 4]);
  } else {
    uint4 o;
    o.x = pack_h2(v[0], v[1]);
    o.y = pack_h2(v[2], v[3]);
    o.z = pack_h2(v[4], v[5]);
    o.w = pack_h2(v[6], v[7]);
    *reinterpret_cast<uint4*>(dst + which * 16) = o;
  }
}

template <int WBITS, bool BF, int GS>
__global__ void __launch_bounds__(256, 2) proj_mma_kernel(const PP p, const uint8_t* xp,
                                                          const float* xsum, const float* xfac) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ __align__(16) uint8_t smraw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wm = warp & 3, wn = warp >> 2;  // 4 x 2 warps: 32 rows x 32 tokens each
  const int M = units_of(p) * p.D;  // rows of every compute unit, unit by unit
  const int m0 = blockIdx.x * kMT, n0 = blockIdx.y * kNT;
  // output row m -> its projection's weights and the weight row
  auto row_w = [&](int m, int64_t& wr) -> const W& {
    const int u = m / p.D;
    int sel, h;
    unit_of(p, u, sel, h);
    wr = (int64_t)h * p.D + (m - u * p.D);
    return w_of(p, sel);
  };
  constexpr int gs = GS;
  const int G = p.hidden / gs;
  constexpr MmaGeo geo{GS, WBITS};
  constexpr int RB = geo.row_bytes(), RP = geo.row_pitch(), KS = geo.ksteps();
  const int64_t row_stride = (int64_t)p.hidden * WBITS / 8;  // bytes per weight row
  auto stage = [&](int b) -> uint8_t* { return smraw + (size_t)b * geo.stage_bytes(); };
  // this thread's weight copies (the same rows for every group): where each
  // row's codes start, worked out once
  constexpr int kCp = (kMT * (RB / 16) + 255) / 256;
  const uint8_t* wsrc[kCp];
  int wdst[kCp];
  bool wok[kCp];
#pragma unroll
  for (int k = 0; k < kCp; k++) {
    const int i = tid + k * 256;
    const int row = i / (RB / 16), c = i - row * (RB / 16);
    const int m = m0 + row;
    wok[k] = i < kMT * (RB / 16) && m < M;
    int64_t wr;
    const W& w = row_w(wok[k] ? m : 0, wr);
    wsrc[k] = reinterpret_cast<const uint8_t*>(w.packed) + wr * row_stride + c * 16;
    wdst[k] = row * RP + c * 16;
  }
  // copies of one group into stage b (every thread commits one cp.async group)
  auto issue = [&](int grp, int b) {
    if (grp < G) {
      uint8_t* st = stage(b);
#pragma unroll
      for (int k = 0; k < kCp; k++)
        if (tid + k * 256 < kMT * (RB / 16))
          cp_async16(st + wdst[k], wsrc[k] + (int64_t)grp * RB, wok[k]);
      uint8_t* sx = st + geo.w_bytes();
      const int nx = KS * kNT * 2;  // 16-byte pieces: 2 per (k-step, token)
      for (int i = tid; i < nx; i += 256) {
        const int s16 = i / (kNT * 2), rem = i - s16 * kNT * 2, n = rem >> 1, half = rem & 1;
        const bool ok = n0 + n < p.R;
        const uint8_t* src = xp + (((int64_t)grp * KS + s16) * p.R + (ok ? n0 + n : 0)) * 32 + half * 16;
        cp_async16(sx + ((size_t)s16 * kNT + n) * 32 + half * 16, src, ok);
      }
      float* ssx = reinterpret_cast<float*>(sx + geo.x_bytes());  // sum(x) [kNT], then 2^e [kNT]
      if (tid < (BF ? 2 : 1) * kNT / 4) {
        const int which = tid / (kNT / 4), n = (tid % (kNT / 4)) * 4;  // 4 tokens per copy
        const int Rp = (p.R + 3) & ~3;  // rows padded to a multiple of 4
        const bool ok = n0 + n < Rp;
        const float* src = which ? xfac : xsum;
        cp_async16(ssx + which * kNT + n, src + (int64_t)grp * Rp + (ok ? n0 + n : 0), ok);
      }
    }
    cp_async_commit();
  };
  float acc[2][4][4], out[2][4][4];
#pragma unroll
  for (int a = 0; a < 2; a++)
#pragma unroll
    for (int b = 0; b < 4; b++)
#pragma unroll
      for (int c = 0; c < 4; c++) acc[a][b][c] = out[a][b][c] = 0.0f;
  // scale (thread < kMT) or bias (thread >= kMT) of one row, one group ahead
  const int srow = tid & (kMT - 1), sm_ = m0 + srow;
  const uint16_t* sbrow = nullptr;
  if (sm_ < M) {
    int64_t wr;
    const W& w = row_w(sm_, wr);
    const uint16_t* src = tid < kMT ? w.scales : w.biases;
    if (src) sbrow = src + wr * G;
  }
  auto fetch_sb = [&](int grp) -> float {
    return (grp < G && sbrow) ? dt_to_f<BF>(__ldg(sbrow + grp)) : 0.0f;
  };
  float sb_next = fetch_sb(0);
#pragma unroll
  for (int s = 0; s < kStages - 1; s++) issue(s, s);
  for (int grp = 0; grp < G; grp++) {
    const int b = grp % kStages;
    uint8_t* st = stage(b);
    float* ssb = reinterpret_cast<float*>(st + geo.w_bytes() + geo.x_bytes() + 2 * kNT * 4);
    ssb[tid] = tid < kMT ? sb_next * 16777216.0f : sb_next;  // scales in the codes' 2^-24 unit
    sb_next = fetch_sb(grp + 1);
    cp_async_wait<kStages - 2>();
    __syncthreads();
    issue(grp + kStages - 1, (grp + kStages - 1) % kStages);
    const uint8_t* sw = st;
    const uint8_t* sx = st + geo.w_bytes();
    const float* ssx = reinterpret_cast<const float*>(sx + geo.x_bytes());
#pragma unroll
    for (int s16 = 0; s16 < KS; s16++) {
      uint32_t a[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; mt++) {
        const int r0 = wm * 32 + mt * 16 + g;
        if (WBITS == 4) {
          const uint2 wa = *reinterpret_cast<const uint2*>(sw + r0 * RP + s16 * 8);
          const uint2 wb = *reinterpret_cast<const uint2*>(sw + (r0 + 8) * RP + s16 * 8);
          a[mt][0] = (wa.x >> (4 * t)) & 0x000F000Fu;
          a[mt][1] = (wb.x >> (4 * t)) & 0x000F000Fu;
          a[mt][2] = (wa.y >> (4 * t)) & 0x000F000Fu;
          a[mt][3] = (wb.y >> (4 * t)) & 0x000F000Fu;
        } else {
          const uint32_t wa = *reinterpret_cast<const uint32_t*>(sw + r0 * RP + s16 * 16 + 4 * t);
          const uint32_t wb = *reinterpret_cast<const uint32_t*>(sw + (r0 + 8) * RP + s16 * 16 + 4 * t);
          a[mt][0] = attn::prmt(wa, 0u, 0x4140u);
          a[mt][1] = attn::prmt(wb, 0u, 0x4140u);
          a[mt][2] = attn::prmt(wa, 0u, 0x4342u);
          a[mt][3] = attn::prmt(wb, 0u, 0x4342u);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; nt++) {
        const int n = wn * 32 + nt * 8 + g;
        const uint2 bf = *reinterpret_cast<const uint2*>(sx + ((size_t)s16 * kNT + n) * 32 + t * 8);
#pragma unroll
        for (int mt = 0; mt < 2; mt++) attn::mma16816(acc[mt][nt], a[mt], bf.x, bf.y);
      }
    }
    // the group's scale and bias, then a fresh dot product
#pragma unroll
    for (int mt = 0; mt < 2; mt++) {
      const int r0 = wm * 32 + mt * 16 + g;
      const float s0 = ssb[r0], s1 = ssb[r0 + 8], b0 = ssb[kMT + r0], b1 = ssb[kMT + r0 + 8];
#pragma unroll
      for (int nt = 0; nt < 4; nt++) {
        const int n = wn * 32 + nt * 8 + 2 * t;
        const float x0 = ssx[n], x1 = ssx[n + 1];
        if (BF) {  // the token blocks' power-of-two input scales back
          const float f0 = ssx[kNT + n], f1 = ssx[kNT + n + 1];
          acc[mt][nt][0] *= f0;
          acc[mt][nt][1] *= f1;
          acc[mt][nt][2] *= f0;
          acc[mt][nt][3] *= f1;
        }
        out[mt][nt][0] = fmaf(s0, acc[mt][nt][0], fmaf(b0, x0, out[mt][nt][0]));
        out[mt][nt][1] = fmaf(s0, acc[mt][nt][1], fmaf(b0, x1, out[mt][nt][1]));
        out[mt][nt][2] = fmaf(s1, acc[mt][nt][2], fmaf(b1, x0, out[mt][nt][2]));
        out[mt][nt][3] = fmaf(s1, acc[mt][nt][3], fmaf(b1, x1, out[mt][nt][3]));
        acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.0f;
      }
    }
  }
  cp_async_wait<0>();
  // the projection rows, f32, in the epilogue's layout part[unit][0][r][d]
#pragma unroll
  for (int mt = 0; mt < 2; mt++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int m = m0 + wm * 32 + mt * 16 + g + 8 * hh;
      if (m >= M) continue;
      const int u = m / p.D, d = m - u * p.D;
      float* dst = p.part + (int64_t)u * p.R * p.D + d;
#pragma unroll
      for (int nt = 0; nt < 4; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int r = n0 + wn * 32 + nt * 8 + 2 * t + e;
          if (r < p.R) dst[(int64_t)r * p.D] = out[mt][nt][2 * hh + e];
        }
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

// Cluster size of the one-launch path on this device: 16 CTAs (a
// non-portable size) where the device can hold such clusters of this
// kernel, else the portable 8; queried once per device.
static int cluster_size(int dev) {
  static std::mutex mu;
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 8;
  std::lock_guard<std::mutex> lk(mu);
  if (cached[dev]) return cached[dev];
  int cs = 8;
  auto kern = proj_cluster_kernel<4, 4, true, 4, 16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(16, 16, 1);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 16 * 1024;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n >= 8) cs = 16;
  }
  cudaGetLastError();  // a refused query leaves no sticky error
  cached[dev] = cs;
  return cs;
}

// Opt `kern` in to 16-CTA clusters on the current device, once per
// (kernel, device): the attribute is per device.
static int32_t allow_wide_clusters(const void* kern) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kern, dev})) return KVQ_OK;
  KVQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  done.insert({kern, dev});
  return KVQ_OK;
}

// The one-launch cluster path: a few rows, every CTA's slice of the hidden
// dimension within kMaxG groups, its inputs within 48 KB of shared memory.
// The projections a call runs (K always; V unless it is K's; Q if given).
static int projections(const ProjArgs& a, const ProjWeights* (&w)[3]) {
  int n = 0;
  w[n++] = &a.wk;
  if (!a.v_from_k) w[n++] = &a.wv;
  if (a.has_q) w[n++] = &a.wq;
  return n;
}
// compute units (heads of the projections run) and finish units (K, V, Q heads)
static int compute_units(const ProjArgs& a, int Hkv) {
  return Hkv + (a.v_from_k ? 0 : Hkv) + (a.has_q ? a.Hq : 0);
}
static int finish_units(const ProjArgs& a, int Hkv) { return 2 * Hkv + (a.has_q ? a.Hq : 0); }

static bool use_cluster(const ProjArgs& a, int cs) {
  const int R = a.B * a.L;
  const ProjWeights* w[3];
  const int n = projections(a, w);
  int gmax = 0, gsmax = 0;
  for (int i = 0; i < n; i++) {
    gmax = std::max(gmax, (a.hidden / w[i]->gs + cs - 1) / cs);
    gsmax = std::max(gsmax, w[i]->gs);
  }
  const int span = gmax * gsmax;
  return R <= 4 && gmax <= kMaxG && (size_t)4 * (256 + kMaxG + span) * 4 <= 48 * 1024;
}

template <int WBITS, int BITS, bool BF, int CS>
static int32_t launch_cluster(const PP& p, int RC, int units, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CS, units, (p.R + RC - 1) / RC);
  cfg.blockDim = dim3(p.D);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  auto k1 = proj_cluster_kernel<WBITS, BITS, BF, 1, CS>;
  auto k4 = proj_cluster_kernel<WBITS, BITS, BF, 4, CS>;
  if (CS > 8) {
    int32_t rc = allow_wide_clusters(reinterpret_cast<const void*>(RC == 1 ? k1 : k4));
    if (rc) return rc;
  }
  KVQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, RC == 1 ? k1 : k4, p));
  return KVQ_OK;
}

template <int WBITS, int BITS>
static int32_t launch_cluster_dt(const PP& p, bool bf, int cs, int RC, int units, size_t smem,
                                 cudaStream_t st) {
  if (cs == 16)
    return bf ? launch_cluster<WBITS, BITS, true, 16>(p, RC, units, smem, st)
              : launch_cluster<WBITS, BITS, false, 16>(p, RC, units, smem, st);
  return bf ? launch_cluster<WBITS, BITS, true, 8>(p, RC, units, smem, st)
            : launch_cluster<WBITS, BITS, false, 8>(p, RC, units, smem, st);
}

// The cluster size of one launch: the device's (16 where it holds such
// clusters), down to 8 when 16-CTA clusters of every compute unit and row
// chunk would not all be resident at once (two CTAs per SM) and 8-CTA
// clusters can take the launch.
static int launch_cluster_size(const ProjArgs& a, int Hkv) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return 8;
  int cs = cluster_size(dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int R = a.B * a.L, chunks = R <= 1 ? 1 : (R + 3) / 4;
  if (cs > 8 && (int64_t)compute_units(a, Hkv) * chunks * cs > 2 * (int64_t)sms &&
      use_cluster(a, 8))
    cs = 8;
  return cs;
}

size_t project_workspace_bytes(const ProjArgs& a, int Hkv, int D, int* splits) {
  const int cs = launch_cluster_size(a, Hkv);
  if (use_cluster(a, cs)) {
    if (splits) *splits = cs;
    return 0;
  }
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int R = a.B * a.L;
  const int G = a.hidden / a.wk.gs;
  const int nrc = (R + proj_rows(R) - 1) / proj_rows(R);
  const int units = compute_units(a, Hkv);
  const ProjWeights* w[3];
  const int n = projections(a, w);
  int gmin = G;
  for (int i = 0; i < n; i++) gmin = std::min(gmin, a.hidden / w[i]->gs);
  int ns = (2 * sms + units * nrc - 1) / (units * nrc);
  ns = std::max(1, std::min(ns, gmin));
  if (splits) *splits = ns;
  // partials (split path; one split on the tensor-core path), then the
  // tensor-core path's fp16 inputs and their group sums
  const size_t part = ((size_t)units * ns * R * D * sizeof(float) + 255) / 256 * 256;
  const size_t xp = ((size_t)R * a.hidden * 2 + 255) / 256 * 256;
  const size_t xs = (size_t)G * ((R + 3) & ~3) * sizeof(float);
  return attn::kPartialOff + part + xp + 2 * xs;  // sums, then the bf16 block scales
}

// proj_epilogue_warp_kernel: one CTA per token, one warp per finish unit.
template <int BITS, bool BF>
static int32_t launch_epilogue_warp_b(const PP& p, cudaStream_t st) {
  const dim3 grid((unsigned)p.R);
  const int fu = 2 * p.Hkv + p.nq;
  const int threads = 32 * fu;
  const size_t smem = (size_t)(fu + 1) * p.D * sizeof(float);
  switch (p.D / 32) {
    case 1: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 1>, grid, dim3(threads), smem, st, p)); break;
    case 2: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 2>, grid, dim3(threads), smem, st, p)); break;
    case 3: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 3>, grid, dim3(threads), smem, st, p)); break;
    case 4: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 4>, grid, dim3(threads), smem, st, p)); break;
    case 5: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 5>, grid, dim3(threads), smem, st, p)); break;
    case 6: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 6>, grid, dim3(threads), smem, st, p)); break;
    case 7: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 7>, grid, dim3(threads), smem, st, p)); break;
    default: KVQ_CUDA_TRY(launch_pdl(proj_epilogue_warp_kernel<BITS, BF, 8>, grid, dim3(threads), smem, st, p)); break;
  }
  return KVQ_OK;
}

static int32_t launch_epilogue_warp(const PP& p, int bits, bool bf, cudaStream_t st) {
  if (bits == 4) return bf ? launch_epilogue_warp_b<4, true>(p, st) : launch_epilogue_warp_b<4, false>(p, st);
  return bf ? launch_epilogue_warp_b<8, true>(p, st) : launch_epilogue_warp_b<8, false>(p, st);
}

int32_t launch_project_append(const ProjArgs& a, int Hkv, RowGeom g, int dtype, TripleView dk,
                              TripleView dv, int64_t dst_row0, void* ws, size_t ws_bytes,
                              cudaStream_t st) {
  const int D = g.D;
  int ns = 1;
  const size_t need = project_workspace_bytes(a, Hkv, D, &ns);
  int32_t rc = KVQ_OK;
  if (need == 0) {
    ws = nullptr;  // the cluster path keeps its partials on chip
  } else if (!ws) {
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
  p.wq = a.has_q ? W{a.wq.packed, static_cast<const uint16_t*>(a.wq.scales),
                      static_cast<const uint16_t*>(a.wq.biases), a.wq.bits, a.wq.gs}
                 : p.wk;
  p.v_from_k = a.v_from_k ? 1 : 0;
  p.Hq = a.has_q ? a.Hq : 0;
  p.nv = a.v_from_k ? 0 : Hkv;
  p.nq = a.has_q ? a.Hq : 0;
  p.q_norm = static_cast<const uint16_t*>(a.q_norm);
  p.q_out = static_cast<uint16_t*>(a.q_out);
  p.R = a.B * a.L;
  p.L = a.L;
  p.hidden = a.hidden;
  p.Hkv = Hkv;
  p.D = D;
  p.ns = ns;
  p.part = ws ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + attn::kPartialOff) : nullptr;
  p.k_norm = static_cast<const uint16_t*>(a.k_norm);
  p.v_norm = static_cast<const uint16_t*>(a.v_norm);
  p.norms = a.norms;
  p.eps = a.eps;
  p.rope_dims = a.rope_dims;
  p.rope_trad = a.rope_traditional ? 1 : 0;
  p.rope_base = a.rope_freqs ? 0.0f : (float)std::log2((double)a.rope_base);
  p.rope_scale = a.rope_scale;
  p.rope_pre = (a.rope_pre_scale == 0.0f || a.rope_pre_scale == 1.0f) ? 0.0f : a.rope_pre_scale;
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
  const ProjWeights* pw[3];
  const int nproj = projections(a, pw);
  bool same_gs = true;
  for (int i = 0; i < nproj; i++) {
    if (pw[i]->bits != a.wk.bits) return fail(KVQ_ERR_ARG, "the projections must share a bit width");
    same_gs = same_gs && pw[i]->gs == a.wk.gs;
  }
  const int units = compute_units(a, Hkv), fu = finish_units(a, Hkv);
  auto block_epilogue = [&]() -> int32_t {
    const dim3 g2(p.R, fu);
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
  };
  const int cs = launch_cluster_size(a, Hkv);
  if (use_cluster(a, cs)) {
    const int RC = p.R <= 1 ? 1 : 4;
    // the largest slice of any projection, in elements
    int span = 0;
    for (int i = 0; i < nproj; i++)
      span = std::max(span, (a.hidden / pw[i]->gs + cs - 1) / cs * pw[i]->gs);
    size_t smem = (size_t)RC * (D + kMaxG + span) * sizeof(float);
    // weight loads per thread beyond the kNB held in registers: staged in
    // shared memory by cp.async before the dependency wait, as many as fit
    // the default 48 KB of dynamic shared memory
    const int e4 = 4 * (32 / a.wk.bits);
    int n4max = 0;
    for (int i = 0; i < nproj; i++)
      n4max = std::max(n4max, (a.hidden / pw[i]->gs + cs - 1) / cs * (pw[i]->gs / e4));
    int nb2 = std::min(std::max(n4max - kNB, 0), kNB2);
    while (nb2 > 0 && smem + (size_t)nb2 * D * 16 > 48 * 1024) nb2--;
    p.nb2 = nb2;
    smem += (size_t)nb2 * D * 16;
    switch ((a.wk.bits == 8 ? 2 : 0) + (g.bits == 8 ? 1 : 0)) {
      case 0: return launch_cluster_dt<4, 4>(p, bf, cs, RC, units, smem, st);
      case 1: return launch_cluster_dt<4, 8>(p, bf, cs, RC, units, smem, st);
      case 2: return launch_cluster_dt<8, 4>(p, bf, cs, RC, units, smem, st);
      default: return launch_cluster_dt<8, 8>(p, bf, cs, RC, units, smem, st);
    }
  }
  // prefill-sized: the tensor-core projection when the projections share a
  // group size and x is 16-byte aligned, then the epilogue
  const bool mma_ok = same_gs && reinterpret_cast<uintptr_t>(a.x) % 16 == 0;
  if (mma_ok) {
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    const size_t part_bytes = ((size_t)units * ns * p.R * D * sizeof(float) + 255) / 256 * 256;
    uint8_t* xp = wsb + attn::kPartialOff + part_bytes;
    float* xsum = reinterpret_cast<float*>(xp + ((size_t)p.R * a.hidden * 2 + 255) / 256 * 256);
    float* xfac = xsum + (size_t)(a.hidden / a.wk.gs) * ((p.R + 3) & ~3);
    p.ns = 1;
    const MmaGeo geo{a.wk.gs, a.wk.bits};
    const int smem = kStages * geo.stage_bytes();
    int dev = 0;
    KVQ_CUDA_TRY(cudaGetDevice(&dev));
    const int64_t nchunks = (int64_t)p.R * (a.hidden / 8);
    const dim3 gx((unsigned)((nchunks + 255) / 256));
    auto xk = [&](auto kern) -> int32_t {
      KVQ_CUDA_TRY(launch_pdl(kern, gx, dim3(256), 0, st, p, xp, xsum, xfac));
      return KVQ_OK;
    };
    rc = a.wk.bits == 4 ? (bf ? xk(proj_xprep_kernel<4, true>) : xk(proj_xprep_kernel<4, false>))
                        : (bf ? xk(proj_xprep_kernel<8, true>) : xk(proj_xprep_kernel<8, false>));
    if (rc) return rc;
    const dim3 gm((units * D + kMT - 1) / kMT, (p.R + kNT - 1) / kNT);
    auto mk = [&](auto kern) -> int32_t {
      int32_t r2 = kernel_setup(reinterpret_cast<const void*>(kern), 256, smem, dev, nullptr);
      if (r2) return r2;
      KVQ_CUDA_TRY(launch_pdl(kern, gm, dim3(256), (size_t)smem, st, p,
                              static_cast<const uint8_t*>(xp), static_cast<const float*>(xsum),
                              static_cast<const float*>(xfac)));
      return KVQ_OK;
    };
    switch ((a.wk.bits == 8 ? 6 : 0) + (bf ? 3 : 0) + (a.wk.gs == 32 ? 0 : a.wk.gs == 64 ? 1 : 2)) {
      case 0: rc = mk(proj_mma_kernel<4, false, 32>); break;
      case 1: rc = mk(proj_mma_kernel<4, false, 64>); break;
      case 2: rc = mk(proj_mma_kernel<4, false, 128>); break;
      case 3: rc = mk(proj_mma_kernel<4, true, 32>); break;
      case 4: rc = mk(proj_mma_kernel<4, true, 64>); break;
      case 5: rc = mk(proj_mma_kernel<4, true, 128>); break;
      case 6: rc = mk(proj_mma_kernel<8, false, 32>); break;
      case 7: rc = mk(proj_mma_kernel<8, false, 64>); break;
      case 8: rc = mk(proj_mma_kernel<8, false, 128>); break;
      case 9: rc = mk(proj_mma_kernel<8, true, 32>); break;
      case 10: rc = mk(proj_mma_kernel<8, true, 64>); break;
      default: rc = mk(proj_mma_kernel<8, true, 128>); break;
    }
    if (rc) return rc;
    // one warp per finish unit while they fit a CTA and its shared memory
    if (fu <= 32 && (size_t)(fu + 1) * D * sizeof(float) <= 48 * 1024)
      return launch_epilogue_warp(p, g.bits, bf, st);
    return block_epilogue();
  }
  const dim3 g1(ns, units, (p.R + proj_rows(p.R) - 1) / proj_rows(p.R));
  const int RC = proj_rows(p.R);
  int wmax = 0;
  for (int i = 0; i < nproj; i++) wmax = std::max(wmax, pw[i]->gs);
  const size_t smem = (size_t)RC * wmax * sizeof(float);
  rc = a.wk.bits == 4 ? (bf ? partial_for<4, true>(RC, g1, threads, smem, st, p)
                            : partial_for<4, false>(RC, g1, threads, smem, st, p))
                      : (bf ? partial_for<8, true>(RC, g1, threads, smem, st, p)
                            : partial_for<8, false>(RC, g1, threads, smem, st, p));
  if (rc) return rc;
  return block_epilogue();
}

}  // namespace kvq
