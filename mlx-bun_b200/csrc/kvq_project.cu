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

#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>

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
  float rope_base, rope_scale, rope_pre;
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
  const uint16_t* wn = sel ? p.v_norm : p.k_norm;
  if ((p.norms & (1 << sel)) && wn) c.wn = dt_to_f<BF>(wn[o]);
  const int half = p.rope_dims / 2;
  if (sel == 0 && o < 2 * half) {
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

// Everything after the projection for one output row (token r) of kv head
// h: `x` is thread o's projected value (the dtype-rounded sum), sel 0 / 1 =
// K / V.  RMSNorm, RoPE (K), the checking copy, then the quantize-on-append.
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
    const uint16_t* wn = sel ? p.v_norm : p.k_norm;
    if (o < D) {
      x = round_dt<BF>(x * n);
      if (wn) x = round_dt<BF>(x * rc.wn);
    }
  }
  if (sel == 0 && p.rope_dims > 0) {
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
  const int r = blockIdx.x, sel = blockIdx.y / p.Hkv, h = blockIdx.y - sel * p.Hkv;
  const int o = threadIdx.x, D = p.D;
  const int src = (sel == 1 && p.v_from_k) ? 0 : sel;
  float x = 0.0f;
  if (o < D) {
    // the split partials, loaded together, summed in split order
    const float* part = p.part + (((int64_t)src * p.Hkv + h) * p.ns * p.R + r) * D + o;
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

// Decode-sized steps (R <= 4 rows): one launch.  A cluster of CS CTAs per
// (K|V, kv head, row chunk) splits the hidden dimension; thread o owns
// output column o.  Each thread first issues everything it will read —
// its weight-row slice (16-byte loads), its group scales and biases, the
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
  extern __shared__ float sm[];  // part[RC][D], sumx[RC][kMaxG], xs[RC][span]
  const int rank = (int)cluster.block_rank();
  const int sel = blockIdx.y / p.Hkv, h = blockIdx.y - sel * p.Hkv;
  const W w = sel ? p.wv : p.wk;
  const int o = threadIdx.x, D = p.D;
  const int G = p.hidden / w.gs, gs = w.gs;
  const int g0 = rank * G / CS, g1 = (rank + 1) * G / CS, ng = g1 - g0;
  const int span = ng * gs;
  float* part = sm;
  float* sumx = sm + RC * D;
  float* xs = sumx + RC * kMaxG;
  const int r0 = blockIdx.z * RC, nr = min(RC, p.R - r0);
  constexpr int PER = 32 / WBITS;
  constexpr int E4 = 4 * PER;            // elements per 16-byte load
  const int u4pg = gs / E4;              // 16-byte loads per group
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
  uint16_t sc16[kMaxG], bi16[kMaxG];
  const uint16_t* sp = w.scales + wrow * G + g0;
  const uint16_t* bp = w.biases ? w.biases + wrow * G + g0 : nullptr;
#pragma unroll
  for (int k = 0; k < kMaxG; k++) {
    sc16[k] = k < ng ? __ldg(sp + k) : (uint16_t)0;
    bi16[k] = (k < ng && bp) ? __ldg(bp + k) : (uint16_t)0;
  }
  RowConsts rcs[RC], rcv[RC];
  if (rank == 0) {
#pragma unroll
    for (int r = 0; r < RC; r++) {
      rcs[r] = row_consts<BF>(p, sel, r0 + r < p.R ? r0 + r : 0);
      rcv[r] = p.v_from_k ? row_consts<BF>(p, 1, r0 + r < p.R ? r0 + r : 0) : rcs[r];
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
    const int k = j / u4pg;
    if (j - k * u4pg == u4pg - 1) {
      uint16_t s16 = sc16[0], b16 = bi16[0];
#pragma unroll
      for (int t = 1; t < kMaxG; t++)
        if (t == k) {
          s16 = sc16[t];
          b16 = bi16[t];
        }
      const float s = dt_to_f<BF>(s16), b = dt_to_f<BF>(b16);
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
  for (int j = kNB; j < n4; j++) consume(__ldg(wp + j), j);
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
    if (p.v_from_k) finish_row<BITS, BF>(p, 1, h, r0 + r, xsum[r], rcv[r], row, red);
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

// The one-launch cluster path: a few rows, every CTA's slice of the hidden
// dimension within kMaxG groups, its inputs within 48 KB of shared memory.
static bool use_cluster(const ProjArgs& a, int cs) {
  const int R = a.B * a.L;
  const int gk = a.hidden / a.wk.gs;
  const int gv = a.v_from_k ? gk : a.hidden / a.wv.gs;
  const int gmax = (std::max(gk, gv) + cs - 1) / cs;
  const int span = gmax * std::max(a.wk.gs, a.v_from_k ? a.wk.gs : a.wv.gs);
  return R <= 4 && gmax <= kMaxG && (size_t)4 * (256 + kMaxG + span) * 4 <= 48 * 1024;
}

template <int WBITS, int BITS, bool BF, int CS>
static int32_t launch_cluster(const PP& p, int RC, int sely, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CS, sely * p.Hkv, (p.R + RC - 1) / RC);
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
    KVQ_CUDA_TRY(cudaFuncSetAttribute(RC == 1 ? k1 : k4,
                                      cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  }
  KVQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, RC == 1 ? k1 : k4, p));
  return KVQ_OK;
}

template <int WBITS, int BITS>
static int32_t launch_cluster_dt(const PP& p, bool bf, int cs, int RC, int sely, size_t smem,
                                 cudaStream_t st) {
  if (cs == 16)
    return bf ? launch_cluster<WBITS, BITS, true, 16>(p, RC, sely, smem, st)
              : launch_cluster<WBITS, BITS, false, 16>(p, RC, sely, smem, st);
  return bf ? launch_cluster<WBITS, BITS, true, 8>(p, RC, sely, smem, st)
            : launch_cluster<WBITS, BITS, false, 8>(p, RC, sely, smem, st);
}

static int current_cluster_size() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 8;
  return cluster_size(dev);
}

size_t project_workspace_bytes(const ProjArgs& a, int Hkv, int D, int* splits) {
  const int cs = current_cluster_size();
  if (use_cluster(a, cs)) {
    if (splits) *splits = cs;
    return 0;
  }
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
  p.v_from_k = a.v_from_k ? 1 : 0;
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
  if (a.wk.bits != (a.v_from_k ? a.wk.bits : a.wv.bits))
    return fail(KVQ_ERR_ARG, "the K and V projections must share a bit width");
  const int cs = current_cluster_size();
  if (use_cluster(a, cs)) {
    const int RC = p.R <= 1 ? 1 : 4;
    // the largest slice of either projection, in elements
    int span = 0;
    for (const ProjWeights* pw : {&a.wk, &a.wv}) {
      if (pw == &a.wv && a.v_from_k) continue;
      span = std::max(span, (a.hidden / pw->gs + cs - 1) / cs * pw->gs);
    }
    const size_t smem = (size_t)RC * (D + kMaxG + span) * sizeof(float);
    const int sely = a.v_from_k ? 1 : 2;
    switch ((a.wk.bits == 8 ? 2 : 0) + (g.bits == 8 ? 1 : 0)) {
      case 0: return launch_cluster_dt<4, 4>(p, bf, cs, RC, sely, smem, st);
      case 1: return launch_cluster_dt<4, 8>(p, bf, cs, RC, sely, smem, st);
      case 2: return launch_cluster_dt<8, 4>(p, bf, cs, RC, sely, smem, st);
      default: return launch_cluster_dt<8, 8>(p, bf, cs, RC, sely, smem, st);
    }
  }
  const dim3 g1(ns, 2 * Hkv, (p.R + proj_rows(p.R) - 1) / proj_rows(p.R));
  const int RC = proj_rows(p.R);
  const int wmax = std::max(a.wk.gs, a.v_from_k ? 0 : a.wv.gs);
  const size_t smem = (size_t)RC * wmax * sizeof(float);
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
