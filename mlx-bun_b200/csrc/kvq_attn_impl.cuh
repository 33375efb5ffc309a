#pragma once
// kvq_attn_impl.cuh — attention over MLX affine-quantized K/V for sm_100a.
//
// Two kernels share the per-slice math:
//   * attn_kernel — a CTA owns one (batch, kv head, block of 8*NT query
//     rows, key split): chunked prefill, windowed decode and debug scores;
//   * attn_bal_kernel — decode over one resident wave of CTAs that split the
//     concatenated key tiles of all (batch, kv head) units evenly, so every
//     SM streams the same bytes whatever the lengths in the batch.
// Query rows are (position, head) pairs of the GQA group (row qr ->
// position qr / nrep, head qr % nrep), so every K/V byte a CTA streams
// serves all query heads that share it.
//
// CTA = W consumer warps + 1 producer warp (warp specialised):
//   * the producer streams the split's key rows in chunks of CH = W*RW rows:
//     six TMA bulk copies (cp.async.bulk, 1-D) per chunk — packed K, K
//     scales, K biases, packed V, V scales, V biases, each a contiguous row
//     range of one (b, h) — into a STAGES-deep shared-memory ring, with one
//     `full` mbarrier (transaction bytes) and one `empty` mbarrier (W
//     consumer arrivals) per stage.  Every wait is bounded: on timeout the
//     kernel raises a device error flag and leaves its loops.
//   * consumer warp w takes rows [w*RW, (w+1)*RW) of every chunk.
// Per consumer slice (RW = 16 or 32 key rows):
//   * a code c becomes the exact fp16 subnormal c * 2^-24 with one logic op
//     per pair (the code's bits in the low mantissa bits, exponent field
//     zero); the tensor cores take subnormal f16 operands exactly, and the
//     2^24 goes into the K scales and the output factor.  Four-bit codes in
//     odd nibbles are taken unshifted (16c) and the factor 16 is folded into
//     the query (K) or the output (V).  Scales and biases are factored out
//     of the inner products
//     (qdot factoring, as in mlx-bun's Metal decode kernel,
//     src/model/fused-decode-kernel.ts:62-114):
//        q . (s*c + b) = s * (q . c) + b * sum(q)
//        sum_n p_n (s_n c_n + b_n) = sum_n (p_n s_n) c_n + sum_n p_n b_n
//   * QK^T: mma.m16n8k16, key rows as M (codes as A, pairs along d), query
//     rows as N (8 per n-tile; q as B, built once per CTA or, in the
//     balanced kernel, once per segment), d as K; one accumulator per
//     quantisation group.
//   * online softmax in f32 with ex2.approx; scores are first rounded to the
//     cache dtype, as the reference graph rounds them
//     (src/model/gemma4-base.ts:1307).
//   * PV: O^T[d x q] += V^T[d x n] (p*s)^T[n x q]; the probability tile goes
//     from the QK accumulator layout to the B-operand layout with one
//     movmatrix.trans per 8x8 block; V codes of a (d, 2 rows) pair are
//     interleaved with one prmt per 16-bit chunk.
//   * splits of the key range merge in fixed order (deterministic): in the
//     split kernel the last CTA to finish, found by an atomic ticket,
//     merges them; the balanced kernel leaves per-warp partials to a merge
//     launch.
//
// Tensor-core choice: decode is HBM-bound with at most 16 query rows per kv
// head, so the register-sourced mma.sync keeps the dequantised codes in
// registers (no shared-memory round trip); tensor throughput is not the
// limit (2 MMAs per key row).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "kvq_internal.h"

namespace kvq {
namespace attn {

constexpr float kNeg = -1.0e30f;             // finite "minus infinity" for masked logits
constexpr float kLog2e = 1.4426950408889634f;
// Lazy rescale: a column's running max moves only when a logit exceeds it
// by more than 4 ln 2, so p <= 16 between updates (p * scale stays far from
// the f16 limit) and most slices skip the reduction and the rescale.
constexpr float kLazyLogit = 2.7725887222397811f;
constexpr int kTile = 16;                     // rows per MMA tile; row-alignment unit
constexpr long long kWaitLimit = 1ll << 30;   // mbarrier polls before declaring a hang
constexpr uint64_t kWaitNs = 2000000000ull;   // ... or 2 s of %globaltimer, whichever first
constexpr int kMergeMax = 64;                 // splits the last CTA merges through shared memory
constexpr int kRowPad = 4;                    // warp-merge rows are D + kRowPad floats apart (bank spread)
constexpr int kBalMinTiles = 8;                // balanced decode: key tiles per CTA at least (one chunk)

struct Params {
  const uint8_t* kp;
  const uint16_t* ks;
  const uint16_t* kb;
  const uint8_t* vp;
  const uint16_t* vs;
  const uint16_t* vb;
  int64_t k_bstride, k_hstride, v_bstride, v_hstride;  // rows
  const uint16_t* q;     // [B, Hq, L, D]
  uint16_t* out;         // [B, Hq, L, D] (mode 0)
  float* pm;             // mode 1 partials [B*Hq]
  float* pl;
  float* po;             // [B*Hq, D]
  float* ws_o;           // split partials
  float* ws_ml;
  unsigned* counters;
  const int32_t* seq_lens;
  int* err;
  float* scores;         // debug: rounded logits [B, Hq, L, N] (nullable)
  int Hq, Hkv, nrep, N, L, QB, rps, nsplit, mode, mask_mode, window;
  float scale;
  int bf16;
  int B;                 // batch entries (balanced kernels)
  int Tu;                // key tiles of a unit of N rows (balanced decode); of one
                         // (b, kv head) pair's query blocks (balanced prefill, whose
                         // CTA count is QB)
};

// ---------------------------------------------------------------- PTX ----

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait; false on timeout (the caller raises the device error flag).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (long long i = 0; i < kWaitLimit; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && global_ns() - t0 > kWaitNs) return false;
  }
  return false;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Codes enter the MMAs as f16 subnormals: value = code * 2^-24.
constexpr float kCodeUnitInv = 16777216.0f;  // 2^24

// 2^x (approximate; flushes results below 2^-126 to zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool BF>
__device__ __forceinline__ float dt_to_f(uint16_t v) {
  if constexpr (BF) return __uint_as_float((uint32_t)v << 16);
  else return __half2float(__ushort_as_half(v));
}

template <bool BF>
__device__ __forceinline__ uint16_t f_to_dt(float f) {
  if constexpr (BF) return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  else return __half_as_ushort(__float2half_rn(f));
}

template <bool BF>
__device__ __forceinline__ float round_dt(float f) {
  if constexpr (BF) return __bfloat162float(__float2bfloat16_rn(f));
  else return __half2float(__float2half_rn(f));
}

// K operand (pairs along d within one row), in units of 2^-24: a 4-bit
// word w holds nibbles e0..e7: x0 = (e0, e4), x1 = 16*(e1, e5), x2 = (e2,
// e6), x3 = 16*(e3, e7); an 8-bit word: x0 = (b0, b1), x1 = (b2, b3).
// (A normal-range form, 1024 + c with the offset cancelled in the
// accumulator, loses ~10 bits of the 4-bit products — enough to flip the
// dtype rounding of large logits; the subnormal form is exact.)
template <int BITS>
__device__ __forceinline__ uint32_t k_extract(uint32_t w, int x) {
  if (BITS == 4) {
    const uint32_t s = (x >= 2) ? (w >> 8) : w;
    const uint32_t m = (x & 1) ? 0x00F000F0u : 0x000F000Fu;
    return s & m;
  } else {
    return prmt(w, 0u, x ? 0x4342u : 0x4140u);
  }
}

// V operand: T holds a 16-bit chunk of row r0 (low half) and of row r1 (high
// half); element j of the chunk as the pair (r0, r1) in units of 2^-24.
template <int BITS>
__device__ __forceinline__ uint32_t v_extract(uint32_t T, int j) {
  if (BITS == 4) {
    const uint32_t s = (j >= 2) ? (T >> 8) : T;
    const uint32_t m = (j & 1) ? 0x00F000F0u : 0x000F000Fu;
    return s & m;
  } else {
    return prmt(T, 0u, j ? 0x4341u : 0x4240u);
  }
}

template <int NBYTES>
__device__ __forceinline__ void lds_words(uint32_t* w, const uint8_t* p) {
  if (NBYTES == 2) {
    w[0] = *reinterpret_cast<const uint16_t*>(p);
  } else if (NBYTES == 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if (NBYTES == 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x;
    w[1] = u.y;
  } else {
#pragma unroll
    for (int i = 0; i < NBYTES / 16; i++) {
      const uint4 u = *reinterpret_cast<const uint4*>(p + 16 * i);
      w[4 * i] = u.x;
      w[4 * i + 1] = u.y;
      w[4 * i + 2] = u.z;
      w[4 * i + 3] = u.w;
    }
  }
}

// All NG scales (or biases) of one row as f32, times `mul` (a power of two).
// Each 32-bit word holds two: converted straight from its halves.
template <int NG, bool BF>
__device__ __forceinline__ void lds_scales(float* out, const uint16_t* row, float mul = 1.0f) {
  uint32_t w[(NG + 1) / 2];
  lds_words<NG * 2>(w, reinterpret_cast<const uint8_t*>(row));
#pragma unroll
  for (int i = 0; i < NG; i++) {
    const uint32_t word = w[i / 2];
    float v;
    if constexpr (BF) {
      v = __uint_as_float((i & 1) ? (word & 0xffff0000u) : (word << 16));
    } else {
      const __half2 h2 = *reinterpret_cast<const __half2*>(&word);
      v = (i & 1) ? __high2float(h2) : __low2float(h2);
    }
    out[i] = v * mul;
  }
}

// Two f32 values rounded to the dtype (one packed conversion).
template <bool BF>
__device__ __forceinline__ void round_dt2(float a, float b, float& ra, float& rb) {
  if constexpr (BF) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(&h);
    ra = __uint_as_float(w << 16);
    rb = __uint_as_float(w & 0xffff0000u);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    ra = __low2float(h);
    rb = __high2float(h);
  }
}

template <int BITS, int D, int GS>
struct Geo {
  static constexpr int NG = D / GS;             // quantisation groups per row
  static constexpr int KRB = D * BITS / 8;      // packed bytes per row
  static constexpr int SRB = NG * 2;            // scale (or bias) bytes per row
  static constexpr int GB = GS * BITS / 8;      // packed bytes per group
  static constexpr int KB = GS * BITS / 32;     // K bytes per lane per (row, group)
  static constexpr int KW = KB / 4;             // ... as words
  static constexpr int E = BITS == 4 ? 4 : 2;   // elements per 16-bit chunk
  static constexpr int C = GS / 8 / E;          // 16-bit V chunks per lane per (row, group)
  static constexpr int VB = 2 * C;              // V bytes per lane per (row, group)
  static constexpr int VW = (VB + 3) / 4;
  static constexpr int MTG = GS / 16;           // PV m-tiles (16 d) per group
  static constexpr int KSTEPS = D / 16;
  static constexpr int MT = D / 16;
  static constexpr int ROWB = 2 * KRB + 4 * SRB;  // bytes per key row (K and V triples)
  static_assert(KB >= 4, "unsupported group size / bits");
};

// Offsets of one ring stage holding CH key rows of the six K/V arrays.
template <int BITS, int D, int GS, int CH>
struct StageLayout {
  using G = Geo<BITS, D, GS>;
  static constexpr int O_KP = 0;
  static constexpr int O_KS = O_KP + CH * G::KRB;
  static constexpr int O_KB = O_KS + CH * G::SRB;
  static constexpr int O_VP = O_KB + CH * G::SRB;
  static constexpr int O_VS = O_VP + CH * G::KRB;
  static constexpr int O_VB = O_VS + CH * G::SRB;
  static constexpr int STAGE = O_VB + CH * G::SRB;
  static_assert((CH * G::SRB) % 16 == 0, "scale rows must tile in 16-byte units");
};

// Shared memory of the split kernel: barriers, merge scratch, then the ring
// (reused as the warp-merge buffer once every stage is consumed).
template <int BITS, int D, int GS, int NT, int W, int RW, int STAGES>
struct Smem {
  using G = Geo<BITS, D, GS>;
  static constexpr int HQ = 8 * NT;
  static constexpr int CH = W * RW;                            // key rows per chunk
  static constexpr int STAGE = StageLayout<BITS, D, GS, CH>::STAGE;
  static constexpr int BARS = 0;                               // full[ST], empty[ST]
  static constexpr int CTRL = BARS + 2 * STAGES * 8;           // ints
  static constexpr int WM = CTRL + 16;                         // f32 [W][HQ] warp maxima
  static constexpr int WL = WM + W * HQ * 4;                   // f32 [W][HQ] warp sums
  static constexpr int RM = WL + W * HQ * 4;                   // f32 [HQ] block maxima
  static constexpr int RL = RM + HQ * 4;                       // f32 [HQ] block sums
  static constexpr int SW = RL + HQ * 4;                       // f32 [HQ][kMergeMax] split m / weights
  static constexpr int SL = SW + HQ * kMergeMax * 4;           // f32 [HQ][kMergeMax] split l
  static constexpr int RA = SL + HQ * kMergeMax * 4;           // f32 [HQ] merge rescale
  static constexpr int STAGES_OFF = (RA + HQ * 4 + 127) / 128 * 128;
  static constexpr int STAGE_BYTES = STAGES * STAGE;
  static constexpr int MERGE_BYTES = W * HQ * (D + kRowPad) * 4;
  static constexpr int TOTAL =
      STAGES_OFF + (STAGE_BYTES > MERGE_BYTES ? STAGE_BYTES : MERGE_BYTES);
};

// Query fragments of one lane group in shared memory: lane l's words at
// uint4 index k*32 + l (conflict-free 16-byte stores and loads).
template <int BITS, int D, int GS, int NT>
struct QFragSlot {
  using G = Geo<BITS, D, GS>;
  static constexpr int NQ = G::KSTEPS * NT * 2;  // qbf words
  static constexpr int NS = NT * G::NG * 2;      // qs_r floats
  static constexpr int W4 = (NQ + NS + 3) / 4;   // uint4 per lane
  static constexpr int BYTES = 32 * W4 * 16;
};

// Shared memory of the balanced kernel: barriers, the per-entry tile table
// (ragged batches), query slots, one query-fragment slot and the ring.
constexpr int kBalMaxBatch = 256;  // ragged batches up to this size use the balanced kernel
template <int BITS, int D, int GS, int NT, int W, int RW, int STAGES>
struct BalSmem {
  using G = Geo<BITS, D, GS>;
  static constexpr int HQ = 8 * NT;
  static constexpr int CH = W * RW;
  static constexpr int STAGE = StageLayout<BITS, D, GS, CH>::STAGE;
  static constexpr int BARS = 0;
  static constexpr int CTRL = BARS + 2 * STAGES * 8;
  static constexpr int BS = CTRL + 16;                          // i64 [B+1] first tile of each entry
  static constexpr int BL = BS + (kBalMaxBatch + 1) * 8;        // int [B] key rows of each entry
  static constexpr int QSLOT = HQ * D * 2;                      // one group's query rows (dtype)
  static constexpr int QS = (BL + kBalMaxBatch * 4 + 127) / 128 * 128;  // [STAGES] query slots
  static constexpr int QF = QS + STAGES * QSLOT;                // second segment's fragments
  static constexpr int STAGES_OFF = (QF + QFragSlot<BITS, D, GS, NT>::BYTES + 127) / 128 * 128;
  static constexpr int TOTAL = STAGES_OFF + STAGES * STAGE;
};

// Running state of one consumer warp.
template <int BITS, int D, int GS, int NT>
struct WarpAcc {
  using G = Geo<BITS, D, GS>;
  float m_run[NT][2], l_run[NT][2], mls_run[NT][2], pb[NT][G::NG][2];
  float o_acc[G::MT][NT][4];
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        m_run[nt][hh] = kNeg;
        mls_run[nt][hh] = kNeg * kLog2e;
        l_run[nt][hh] = 0.0f;
#pragma unroll
        for (int grp = 0; grp < G::NG; grp++) pb[nt][grp][hh] = 0.0f;
      }
#pragma unroll
    for (int mt = 0; mt < G::MT; mt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int c = 0; c < 4; c++) o_acc[mt][nt][c] = 0.0f;
  }
};

// Query operand of one consumer lane (the B operand of QK).
template <int BITS, int D, int GS, int NT>
struct QFrag {
  using G = Geo<BITS, D, GS>;
  uint32_t qbf[G::KSTEPS][NT][2];
  float qs_r[NT][G::NG][2];
};

// d positions of the query halves that fragment word (kk, w2) of lane t
// pairs with the K codes, and the factor folded into them (1/16 for the
// odd nibbles of 4-bit codes, which the K fragments take as 16c).
template <int BITS, int GS>
__device__ __forceinline__ void q_positions(int kk, int w2, int t, int mtg, int& d_lo, int& d_hi,
                                            float& fac) {
  const int grp = kk / mtg, kin = kk % mtg, v = 2 * kin + w2;
  fac = 1.0f;
  if (BITS == 4) {
    const int wi = v / 4, x = v % 4;
    const int base = grp * GS + t * (GS / 4) + 8 * wi;
    d_lo = base + x;
    d_hi = base + x + 4;
    if (x & 1) fac = 0.0625f;
  } else {
    const int wi = v / 2, x = v % 2;
    const int base = grp * GS + t * (GS / 4) + 4 * wi;
    d_lo = base + 2 * x;
    d_hi = base + 2 * x + 1;
  }
}

// A lane's raw query halves (dtype bits, lo | hi << 16 per fragment word),
// zero for rows past qrows.  qs: the group's query rows in shared memory
// ([nrep][D], L = 1), or nullptr to read them from global memory.
template <int BITS, int D, int GS, int NT>
struct QRaw {
  uint32_t w[NT][Geo<BITS, D, GS>::KSTEPS][2];
};

template <int BITS, int D, int GS, int NT>
__device__ __forceinline__ void load_qraw(QRaw<BITS, D, GS, NT>& r, const Params& p, int b,
                                          int kvh, int qr0, int qrows, int g, int t,
                                          const uint16_t* qs = nullptr) {
  using G = Geo<BITS, D, GS>;
  const int nrep = p.nrep, L = p.L;
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int qr = qr0 + nt * 8 + g;
    const bool qvalid = qr < qrows;
    const int l = qvalid ? qr / nrep : 0, hh = qvalid ? qr - l * nrep : 0;
    const uint16_t* qrow =
        qs ? qs + hh * D : p.q + (((int64_t)b * p.Hq + kvh * nrep + hh) * L + l) * D;
#pragma unroll
    for (int kk = 0; kk < G::KSTEPS; kk++)
#pragma unroll
      for (int w2 = 0; w2 < 2; w2++) {
        int d_lo, d_hi;
        float fac;
        q_positions<BITS, GS>(kk, w2, t, G::MTG, d_lo, d_hi, fac);
        const uint32_t h0 = qvalid ? (qs ? qrow[d_lo] : __ldg(qrow + d_lo)) : 0u;
        const uint32_t h1 = qvalid ? (qs ? qrow[d_hi] : __ldg(qrow + d_hi)) : 0u;
        r.w[nt][kk][w2] = h0 | (h1 << 16);
      }
  }
}

// Lane (g, t) holds q * dtype(scale) (rounded to dtype, like mulScalar) of
// query row qr0 + nt*8 + g at the d positions its K fragments pair with;
// sum(q) per group comes from the 4 lanes t of the row, then moves to the
// lanes that own each column of the score tile.
template <int BITS, int D, int GS, int NT, bool BF>
__device__ __forceinline__ void qfrag_from_raw(QFrag<BITS, D, GS, NT>& f,
                                               const QRaw<BITS, D, GS, NT>& r, const Params& p,
                                               int t) {
  using G = Geo<BITS, D, GS>;
  const float scale_dt = round_dt<BF>(p.scale);
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    float gsum[G::NG];
#pragma unroll
    for (int grp = 0; grp < G::NG; grp++) gsum[grp] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < G::KSTEPS; kk++)
#pragma unroll
      for (int w2 = 0; w2 < 2; w2++) {
        int d_lo, d_hi;
        float fac;
        q_positions<BITS, GS>(kk, w2, t, G::MTG, d_lo, d_hi, fac);
        const uint32_t hw = r.w[nt][kk][w2];
        // zero halves (rows past qrows) stay zero
        const float a0 = round_dt<BF>(dt_to_f<BF>((uint16_t)(hw & 0xffffu)) * scale_dt);
        const float a1 = round_dt<BF>(dt_to_f<BF>((uint16_t)(hw >> 16)) * scale_dt);
        gsum[kk / G::MTG] += a0 + a1;
        f.qbf[kk][nt][w2] = pack_h2(a0 * fac, a1 * fac);
      }
#pragma unroll
    for (int grp = 0; grp < G::NG; grp++) {
      float v = gsum[grp];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      // column 2t + hh of this n-tile is query row nt*8 + 2t + hh, held by lanes g = 2t + hh
      f.qs_r[nt][grp][0] = __shfl_sync(0xffffffffu, v, (2 * t) << 2);
      f.qs_r[nt][grp][1] = __shfl_sync(0xffffffffu, v, (2 * t + 1) << 2);
    }
  }
}

template <int BITS, int D, int GS, int NT, bool BF>
__device__ __forceinline__ void load_qfrag(QFrag<BITS, D, GS, NT>& f, const Params& p, int b,
                                           int kvh, int qr0, int qrows, int g, int t,
                                           const uint16_t* qs = nullptr) {
  QRaw<BITS, D, GS, NT> r;
  load_qraw<BITS, D, GS, NT>(r, p, b, kvh, qr0, qrows, g, t, qs);
  qfrag_from_raw<BITS, D, GS, NT, BF>(f, r, p, t);
}

template <int BITS, int D, int GS, int NT>
__device__ __forceinline__ void store_qfrag(const QFrag<BITS, D, GS, NT>& f, uint8_t* slot,
                                            int lane) {
  using QS = QFragSlot<BITS, D, GS, NT>;
  uint32_t w[QS::W4 * 4];
  const uint32_t* qb = &f.qbf[0][0][0];
  const float* qs = &f.qs_r[0][0][0];
#pragma unroll
  for (int k = 0; k < QS::W4 * 4; k++)
    w[k] = k < QS::NQ ? qb[k] : (k < QS::NQ + QS::NS ? __float_as_uint(qs[k - QS::NQ]) : 0u);
#pragma unroll
  for (int k = 0; k < QS::W4; k++)
    *reinterpret_cast<uint4*>(slot + (k * 32 + lane) * 16) =
        make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
}

template <int BITS, int D, int GS, int NT>
__device__ __forceinline__ void load_qfrag_slot(QFrag<BITS, D, GS, NT>& f, const uint8_t* slot,
                                                int lane) {
  using QS = QFragSlot<BITS, D, GS, NT>;
  uint32_t w[QS::W4 * 4];
#pragma unroll
  for (int k = 0; k < QS::W4; k++) {
    const uint4 v = *reinterpret_cast<const uint4*>(slot + (k * 32 + lane) * 16);
    w[4 * k] = v.x;
    w[4 * k + 1] = v.y;
    w[4 * k + 2] = v.z;
    w[4 * k + 3] = v.w;
  }
  uint32_t* qb = &f.qbf[0][0][0];
  float* qs = &f.qs_r[0][0][0];
#pragma unroll
  for (int k = 0; k < QS::NQ; k++) qb[k] = w[k];
#pragma unroll
  for (int k = 0; k < QS::NS; k++) qs[k] = __uint_as_float(w[QS::NQ + k]);
}

// Key-index limits (inclusive) of this lane's query columns.
template <int NT>
__device__ __forceinline__ void column_bounds(int (&klo)[NT][2], int (&khi)[NT][2],
                                              const Params& p, int qr0, int qrows, int Nb, int t) {
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int qr = qr0 + nt * 8 + 2 * t + hh;
      int a = 0, z = Nb - 1;
      if (p.mask_mode == 1 && qr < qrows) {
        const int pos = Nb - p.L + qr / p.nrep;
        z = min(z, pos);
        if (p.window > 0) a = max(0, pos - p.window + 1);
      }
      klo[nt][hh] = a;
      khi[nt][hh] = z;
    }
}

// One consumer slice: RW key rows of the stage at `st` (chunk rows r_base..,
// global key rows srow0..), valid below n1; `fast` = every row valid for
// every column (no masking work).
template <int BITS, int D, int GS, int NT, int RW, int CH, bool BF, bool FAST>
__device__ __forceinline__ void process_slice(WarpAcc<BITS, D, GS, NT>& A,
                                              const QFrag<BITS, D, GS, NT>& Q, const Params& p,
                                              const uint8_t* st, int r_base, int srow0, int n1,
                                              const int (&klo)[NT][2],
                                              const int (&khi)[NT][2], int qr0, int qrows,
                                              int kvh, int b, int g, int t) {
  constexpr bool fast = FAST;
  using G = Geo<BITS, D, GS>;
  using Lay = StageLayout<BITS, D, GS, CH>;
  constexpr int MTS = RW / 16;  // 16-row m-tiles per consumer slice
  const int nrep = p.nrep, L = p.L;
  auto& m_run = A.m_run;
  auto& l_run = A.l_run;
  auto& mls_run = A.mls_run;
  auto& pb = A.pb;
  auto& o_acc = A.o_acc;
  const auto& qbf = Q.qbf;
  const auto& qs_r = Q.qs_r;
  // ---------------- scores ----------------
  float sc[MTS][NT][4];
#pragma unroll
  for (int mt = 0; mt < MTS; mt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int cc = 0; cc < 4; cc++) sc[mt][nt][cc] = 0.0f;
#pragma unroll
  for (int mt = 0; mt < MTS; mt++) {
    const int R0 = r_base + mt * 16 + g, R1 = R0 + 8;
    float ks0[G::NG], kb0[G::NG], ks1[G::NG], kb1[G::NG];
    lds_scales<G::NG, BF>(ks0, reinterpret_cast<const uint16_t*>(st + Lay::O_KS) + R0 * G::NG,
                          kCodeUnitInv);
    lds_scales<G::NG, BF>(kb0, reinterpret_cast<const uint16_t*>(st + Lay::O_KB) + R0 * G::NG);
    lds_scales<G::NG, BF>(ks1, reinterpret_cast<const uint16_t*>(st + Lay::O_KS) + R1 * G::NG,
                          kCodeUnitInv);
    lds_scales<G::NG, BF>(kb1, reinterpret_cast<const uint16_t*>(st + Lay::O_KB) + R1 * G::NG);
#pragma unroll
    for (int grp = 0; grp < G::NG; grp++) {
      uint32_t kw0[G::KW], kw1[G::KW];
      lds_words<G::KB>(kw0, st + Lay::O_KP + R0 * G::KRB + grp * G::GB + t * G::KB);
      lds_words<G::KB>(kw1, st + Lay::O_KP + R1 * G::KRB + grp * G::GB + t * G::KB);
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
      }
#pragma unroll
      for (int kin = 0; kin < G::MTG; kin++) {
        uint32_t a[4];
#pragma unroll
        for (int w2 = 0; w2 < 2; w2++) {
          const int v = 2 * kin + w2;
          const int wi = BITS == 4 ? v / 4 : v / 2;
          const int x = BITS == 4 ? v % 4 : v % 2;
          a[2 * w2] = k_extract<BITS>(kw0[wi], x);
          a[2 * w2 + 1] = k_extract<BITS>(kw1[wi], x);
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
          mma16816(acc[nt], a, qbf[grp * G::MTG + kin][nt][0],
                   qbf[grp * G::MTG + kin][nt][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        // s += ks * acc + kb * sum(q), two query columns per paired fp32 op
        const float2 qs2 = make_float2(qs_r[nt][grp][0], qs_r[nt][grp][1]);
        float2 s01 = make_float2(sc[mt][nt][0], sc[mt][nt][1]);
        float2 s23 = make_float2(sc[mt][nt][2], sc[mt][nt][3]);
        s01 = __ffma2_rn(make_float2(kb0[grp], kb0[grp]), qs2, s01);
        s23 = __ffma2_rn(make_float2(kb1[grp], kb1[grp]), qs2, s23);
        s01 = __ffma2_rn(make_float2(ks0[grp], ks0[grp]), make_float2(acc[nt][0], acc[nt][1]), s01);
        s23 = __ffma2_rn(make_float2(ks1[grp], ks1[grp]), make_float2(acc[nt][2], acc[nt][3]), s23);
        sc[mt][nt][0] = s01.x;
        sc[mt][nt][1] = s01.y;
        sc[mt][nt][2] = s23.x;
        sc[mt][nt][3] = s23.y;
      }
    }
  }

  // ---------------- online softmax ----------------
  // Logits rounded to the dtype, masked to kNeg.  When no lane sees a
  // logit above its column's running max (most slices once a few have
  // passed) the max, and so every scale factor, is unchanged: skip the
  // cross-lane reduction and the rescale.  Otherwise do the full update.
  float pr[MTS][NT][4];
  float alpha[NT][2];
  bool rescale = false;
  float x[NT][2][MTS][2];
  bool vv[NT][2][MTS][2];
  bool above = false;
  float rsc[MTS][NT][4];  // logits rounded to the dtype, two per conversion
#pragma unroll
  for (int mt = 0; mt < MTS; mt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      round_dt2<BF>(sc[mt][nt][0], sc[mt][nt][1], rsc[mt][nt][0], rsc[mt][nt][1]);
      round_dt2<BF>(sc[mt][nt][2], sc[mt][nt][3], rsc[mt][nt][2], rsc[mt][nt][3]);
    }
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++)
#pragma unroll
      for (int mt = 0; mt < MTS; mt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int r = srow0 + mt * 16 + g + 8 * e;
          const float rs = rsc[mt][nt][2 * e + hh];
          if (fast) {
            vv[nt][hh][mt][e] = true;
            x[nt][hh][mt][e] = rs;
          } else {
            vv[nt][hh][mt][e] = r < n1 && r >= klo[nt][hh] && r <= khi[nt][hh];
            x[nt][hh][mt][e] = vv[nt][hh][mt][e] ? rs : kNeg;
            if (p.scores && vv[nt][hh][mt][e]) {
              const int qr = qr0 + nt * 8 + 2 * t + hh;
              if (qr < qrows) {
                const int l = qr / nrep, hq = kvh * nrep + (qr - l * nrep);
                p.scores[(((int64_t)b * p.Hq + hq) * L + l) * p.N + r] = rs;
              }
            }
          }
          above |= x[nt][hh][mt][e] > m_run[nt][hh] + kLazyLogit;
        }
  const bool rescale_all = __any_sync(0xffffffffu, above);
  if (rescale_all) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        float tm = x[nt][hh][0][0];
#pragma unroll
        for (int mt = 0; mt < MTS; mt++)
#pragma unroll
          for (int e = 0; e < 2; e++) tm = fmaxf(tm, x[nt][hh][mt][e]);
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 4));
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 8));
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
        const float mn = fmaxf(m_run[nt][hh], tm);
        // (m_old - m_new) first: exactly 0 when the max is unchanged, even at
        // the -1e30 sentinel (an fma against the rounded product would leave
        // its rounding residual, ~1e23 there, and 2^that is inf).
        const float al = ex2((m_run[nt][hh] - mn) * kLog2e);
        rescale |= (mn != m_run[nt][hh]);
        alpha[nt][hh] = al;
        m_run[nt][hh] = mn;
        mls_run[nt][hh] = mn * kLog2e;
      }
    }
  }
  // p = 2^(x log2e - m log2e) for both columns of a lane at once (paired
  // fp32 ops); the lazy path keeps l, the update path rescales it by alpha
  {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const float2 nm = make_float2(-mls_run[nt][0], -mls_run[nt][1]);
      float2 lsum = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int mt = 0; mt < MTS; mt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const float2 arg = __ffma2_rn(make_float2(x[nt][0][mt][e], x[nt][1][mt][e]),
                                        make_float2(kLog2e, kLog2e), nm);
          float2 pv = make_float2(ex2(arg.x), ex2(arg.y));
          if (!fast) {
            pv.x = vv[nt][0][mt][e] ? pv.x : 0.0f;
            pv.y = vv[nt][1][mt][e] ? pv.y : 0.0f;
          }
          pr[mt][nt][2 * e] = pv.x;
          pr[mt][nt][2 * e + 1] = pv.y;
          lsum = __fadd2_rn(lsum, pv);
        }
      if (rescale_all) {
        l_run[nt][0] = fmaf(l_run[nt][0], alpha[nt][0], lsum.x);
        l_run[nt][1] = fmaf(l_run[nt][1], alpha[nt][1], lsum.y);
      } else {
        l_run[nt][0] += lsum.x;
        l_run[nt][1] += lsum.y;
      }
    }
  }
  if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
      for (int mt = 0; mt < G::MT; mt++) {
        o_acc[mt][nt][0] *= alpha[nt][0];
        o_acc[mt][nt][1] *= alpha[nt][1];
        o_acc[mt][nt][2] *= alpha[nt][0];
        o_acc[mt][nt][3] *= alpha[nt][1];
      }
#pragma unroll
      for (int grp = 0; grp < G::NG; grp++) {
        pb[nt][grp][0] *= alpha[nt][0];
        pb[nt][grp][1] *= alpha[nt][1];
      }
    }
  }

  // ---------------- P V ----------------
#pragma unroll
  for (int kk = 0; kk < MTS; kk++) {  // 16-row k-steps of the slice
    const int R0 = r_base + kk * 16 + g, R1 = R0 + 8;
    float vs0[G::NG], vb0[G::NG], vs1[G::NG], vb1[G::NG];
    lds_scales<G::NG, BF>(vs0, reinterpret_cast<const uint16_t*>(st + Lay::O_VS) + R0 * G::NG);
    lds_scales<G::NG, BF>(vb0, reinterpret_cast<const uint16_t*>(st + Lay::O_VB) + R0 * G::NG);
    lds_scales<G::NG, BF>(vs1, reinterpret_cast<const uint16_t*>(st + Lay::O_VS) + R1 * G::NG);
    lds_scales<G::NG, BF>(vb1, reinterpret_cast<const uint16_t*>(st + Lay::O_VB) + R1 * G::NG);
    const int vr = r_base + kk * 16 + 2 * t;
#pragma unroll
    for (int grp = 0; grp < G::NG; grp++) {
      uint32_t bfr[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        // p == 0 for masked rows: select, never multiply stale scales.
        const float p0 = pr[kk][nt][0], p1 = pr[kk][nt][1], p2 = pr[kk][nt][2],
                    p3 = pr[kk][nt][3];
        float q0, q1, q2, q3;
        if (fast) {  // paired fp32 ops: the two query columns of a lane
          float2 pbv = make_float2(pb[nt][grp][0], pb[nt][grp][1]);
          pbv = __ffma2_rn(make_float2(p2, p3), make_float2(vb1[grp], vb1[grp]), pbv);
          pbv = __ffma2_rn(make_float2(p0, p1), make_float2(vb0[grp], vb0[grp]), pbv);
          pb[nt][grp][0] = pbv.x;
          pb[nt][grp][1] = pbv.y;
          const float2 q01 = __fmul2_rn(make_float2(p0, p1), make_float2(vs0[grp], vs0[grp]));
          const float2 q23 = __fmul2_rn(make_float2(p2, p3), make_float2(vs1[grp], vs1[grp]));
          q0 = q01.x;
          q1 = q01.y;
          q2 = q23.x;
          q3 = q23.y;
        } else {
          pb[nt][grp][0] += (p0 != 0.0f ? p0 * vb0[grp] : 0.0f) + (p2 != 0.0f ? p2 * vb1[grp] : 0.0f);
          pb[nt][grp][1] += (p1 != 0.0f ? p1 * vb0[grp] : 0.0f) + (p3 != 0.0f ? p3 * vb1[grp] : 0.0f);
          q0 = p0 != 0.0f ? p0 * vs0[grp] : 0.0f;
          q1 = p1 != 0.0f ? p1 * vs0[grp] : 0.0f;
          q2 = p2 != 0.0f ? p2 * vs1[grp] : 0.0f;
          q3 = p3 != 0.0f ? p3 * vs1[grp] : 0.0f;
        }
        bfr[nt][0] = movmatrix_t(pack_h2(q0, q1));
        bfr[nt][1] = movmatrix_t(pack_h2(q2, q3));
      }
      uint32_t vw[4][G::VW];
      const uint8_t* vrow = st + Lay::O_VP + grp * G::GB + g * G::VB;
      lds_words<G::VB>(vw[0], vrow + (vr)*G::KRB);
      lds_words<G::VB>(vw[1], vrow + (vr + 1) * G::KRB);
      lds_words<G::VB>(vw[2], vrow + (vr + 8) * G::KRB);
      lds_words<G::VB>(vw[3], vrow + (vr + 9) * G::KRB);
      uint32_t af[G::MTG][4];
#pragma unroll
      for (int cc = 0; cc < G::C; cc++) {
        const uint32_t sel = (cc & 1) ? 0x7632u : 0x5410u;
        const uint32_t Tlo = prmt(vw[0][cc / 2], vw[1][cc / 2], sel);
        const uint32_t Thi = prmt(vw[2][cc / 2], vw[3][cc / 2], sel);
#pragma unroll
        for (int j = 0; j < G::E; j++) {
          const int sl = cc * G::E + j;
          const int mt = sl % G::MTG, half = sl / G::MTG;
          af[mt][half] = v_extract<BITS>(Tlo, j);      // a0 (m-row g) / a1 (m-row g+8)
          af[mt][2 + half] = v_extract<BITS>(Thi, j);  // a2 / a3
        }
      }
#pragma unroll
      for (int mt = 0; mt < G::MTG; mt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
          mma16816(o_acc[grp * G::MTG + mt][nt], af[mt], bfr[nt][0], bfr[nt][1]);
    }
  }
}

// process_slice with the full-slice flag as a compile-time branch.
template <int BITS, int D, int GS, int NT, int RW, int CH, bool BF>
__device__ __forceinline__ void run_slice(WarpAcc<BITS, D, GS, NT>& A,
                                          const QFrag<BITS, D, GS, NT>& Q, const Params& p,
                                          const uint8_t* st, int r_base, int srow0, int n1,
                                          bool fast, const int (&klo)[NT][2],
                                          const int (&khi)[NT][2], int qr0, int qrows, int kvh,
                                          int b, int g, int t) {
  if (fast)
    process_slice<BITS, D, GS, NT, RW, CH, BF, true>(A, Q, p, st, r_base, srow0, n1, klo, khi, qr0,
                                                     qrows, kvh, b, g, t);
  else
    process_slice<BITS, D, GS, NT, RW, CH, BF, false>(A, Q, p, st, r_base, srow0, n1, klo, khi,
                                                      qr0, qrows, kvh, b, g, t);
}

// Row-lane reductions of l and the bias sums at the end of a warp's work.
template <int BITS, int D, int GS, int NT>
__device__ __forceinline__ void warp_reduce(WarpAcc<BITS, D, GS, NT>& A) {
  using G = Geo<BITS, D, GS>;
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      float l = A.l_run[nt][hh];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      A.l_run[nt][hh] = l;
#pragma unroll
      for (int grp = 0; grp < G::NG; grp++) {
        float v = A.pb[nt][grp][hh];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        A.pb[nt][grp][hh] = v;
      }
    }
}

// Rescale a warp's partial to the block maxima (from wm) so the cross-warp
// combine is a plain sum; lanes g == 0 publish l (wl) and warp 0 the maxima (rm).
template <int BITS, int D, int GS, int NT, int W>
__device__ __forceinline__ void rescale_warp(WarpAcc<BITS, D, GS, NT>& A, const float* wm,
                                             float* wl, float* rm, int warp, int g, int t) {
  using G = Geo<BITS, D, GS>;
  constexpr int HQ = 8 * NT;
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int col = nt * 8 + 2 * t + hh;
      float M = wm[col];
#pragma unroll
      for (int w = 1; w < W; w++) M = fmaxf(M, wm[w * HQ + col]);
      const float f = ex2((A.m_run[nt][hh] - M) * kLog2e);
      A.l_run[nt][hh] *= f;
#pragma unroll
      for (int grp = 0; grp < G::NG; grp++) A.pb[nt][grp][hh] *= f;
#pragma unroll
      for (int mtg = 0; mtg < G::MT; mtg++) {
        A.o_acc[mtg][nt][hh] *= f;
        A.o_acc[mtg][nt][2 + hh] *= f;
      }
      if (g == 0) {
        wl[warp * HQ + col] = A.l_run[nt][hh];
        if (warp == 0) rm[col] = M;
      }
    }
}

// Write (or add) a warp's output partial o * fac + sum(p * bias) into wo
// [HQ][D + kRowPad].  A lane holds GS/8 consecutive d of each (group,
// column), stored as 16-byte vectors; with the padded row stride a warp's
// vector store meets at most 2-way bank conflicts.
template <int BITS, int D, int GS, int NT, bool ADD>
__device__ __forceinline__ void store_warp(const WarpAcc<BITS, D, GS, NT>& A, float* wo, int g,
                                           int t) {
  using G = Geo<BITS, D, GS>;
  constexpr int MS = D + kRowPad;
  constexpr int V = GS / 8;  // consecutive d per lane per (group, column): d = grp*GS + g*V + sl
  static_assert(V == G::C * G::E && V == 2 * G::MTG && V % 4 == 0, "lane d layout");
#pragma unroll
  for (int grp = 0; grp < G::NG; grp++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        float v[V];
#pragma unroll
        for (int sl = 0; sl < V; sl++) {
          const int mt = sl % G::MTG, half = sl / G::MTG;
          const float fac = (BITS == 4 && (mt & 1)) ? kCodeUnitInv * 0.0625f : kCodeUnitInv;
          v[sl] = fmaf(A.o_acc[grp * G::MTG + mt][nt][half * 2 + hh], fac, A.pb[nt][grp][hh]);
        }
        float* dst = wo + (nt * 8 + 2 * t + hh) * MS + grp * GS + g * V;
#pragma unroll
        for (int q4 = 0; q4 < V / 4; q4++) {
          float4* p4 = reinterpret_cast<float4*>(dst + 4 * q4);
          float4 x = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
          if (ADD) {
            const float4 y = *p4;
            x.x += y.x;
            x.y += y.y;
            x.z += y.z;
            x.w += y.w;
          }
          *p4 = x;
        }
      }
}

// One output element of query row `orow`: the normalised result (mode 0) or
// the unnormalised partial with its (m, l) (mode 1).
template <int D, bool BF>
__device__ __forceinline__ void write_row(const Params& p, int64_t orow, int d, float O, float M,
                                          float Lsum) {
  if (p.mode == 0) {
    p.out[orow * D + d] = f_to_dt<BF>(Lsum > 0.0f ? O / Lsum : 0.0f);
  } else {
    p.po[orow * D + d] = O;
    if (d == 0) {
      p.pm[orow] = M;
      p.pl[orow] = Lsum;
    }
  }
}

// Barrier among the first `nthreads` threads of the CTA (barrier 1; the
// kernels use barrier 0 only through __syncthreads).
__device__ __forceinline__ void bar_sync1(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Merge the partials (m, l, o) that `nseg` key ranges wrote to consecutive
// slots slot0.. of the workspace (HQ rows each; rows [0, rows) are live) and
// write each live row through row_of(r): o = sum_j o_j e^(m_j - M) /
// sum_j l_j e^(m_j - M), M = max_j m_j, summed in j order (deterministic).
// Run by threads [0, NTH) together.  Every (m, l) is fetched in one round of
// loads into shared memory, and the o sums issue their loads in batches, so
// the merge pays a few L2 round trips rather than one per range.
template <int D, int HQ, int NTH, bool BF, class RowOf>
__device__ __forceinline__ void merge_slots(const Params& p, int64_t slot0, int nseg, int rows,
                                            float* sm, float* sl, float* rm, float* rl,
                                            float* ra, float* carry, int tid, RowOf row_of) {
  constexpr int KB = 4;  // output elements whose loads are batched together
  const int live = rows * D;
  for (int j0 = 0; j0 < nseg; j0 += kMergeMax) {
    const int nj = min(kMergeMax, nseg - j0);
    const bool last = j0 + nj >= nseg;
    if (j0) bar_sync1(NTH);  // the previous pass is done with sm / ra / carry
    for (int e = tid; e < nj * rows; e += NTH) {
      const int j = e / rows, r = e - j * rows;
      const float* ml = p.ws_ml + ((slot0 + j0 + j) * HQ + r) * 2;
      sm[r * kMergeMax + j] = __ldcg(ml);
      sl[r * kMergeMax + j] = __ldcg(ml + 1);
    }
    bar_sync1(NTH);
    if (tid < rows) {
      const int r = tid;
      const float Mo = j0 ? rm[r] : kNeg;
      float M = Mo;
      for (int j = 0; j < nj; j++) M = fmaxf(M, sm[r * kMergeMax + j]);
      const float a = ex2((Mo - M) * kLog2e);
      float L = j0 ? rl[r] * a : 0.0f;
      for (int j = 0; j < nj; j++) {
        const float w = ex2((sm[r * kMergeMax + j] - M) * kLog2e);
        sm[r * kMergeMax + j] = w;
        L = fmaf(sl[r * kMergeMax + j], w, L);
      }
      rm[r] = M;
      rl[r] = L;
      ra[r] = a;
    }
    bar_sync1(NTH);
    // output elements e = tid + k*NTH, KB of them at a time (a sum carried
    // between passes waits in `carry`)
#pragma unroll 1
    for (int e0 = tid; e0 < live; e0 += KB * NTH) {
      float acc[KB];
      int rr[KB];
      const float* src[KB];
      bool ok[KB];
#pragma unroll
      for (int kb = 0; kb < KB; kb++) {
        const int e = e0 + kb * NTH;
        ok[kb] = e < live;
        const int r = ok[kb] ? e / D : 0, d = ok[kb] ? e - r * D : 0;
        rr[kb] = r;
        src[kb] = p.ws_o + ((slot0 + j0) * HQ + r) * D + d;
        acc[kb] = (ok[kb] && j0) ? carry[e] * ra[r] : 0.0f;
      }
      for (int j = 0; j < nj; j += 4) {
        float v[KB][4];
#pragma unroll
        for (int kb = 0; kb < KB; kb++)
#pragma unroll
          for (int jj = 0; jj < 4; jj++)
            v[kb][jj] = (ok[kb] && j + jj < nj) ? __ldcg(src[kb] + (int64_t)(j + jj) * HQ * D) : 0.0f;
#pragma unroll
        for (int kb = 0; kb < KB; kb++)
#pragma unroll
          for (int jj = 0; jj < 4; jj++)
            if (j + jj < nj) acc[kb] = fmaf(v[kb][jj], sm[rr[kb] * kMergeMax + j + jj], acc[kb]);
      }
#pragma unroll
      for (int kb = 0; kb < KB; kb++) {
        const int e = e0 + kb * NTH;
        if (!ok[kb]) continue;
        if (last) write_row<D, BF>(p, row_of(rr[kb]), e - rr[kb] * D, acc[kb], rm[rr[kb]], rl[rr[kb]]);
        else carry[e] = acc[kb];
      }
    }
  }
}

// Issue the six bulk copies of `rows` (a multiple of 16) key rows starting
// at row `row` of the (b, h) pair whose first rows are kbase / vbase.
// With q_dst, also copy q_bytes of query rows from q_src (the first chunk
// of a segment after the second carries its query group).
template <int BITS, int D, int GS, int CH>
__device__ __forceinline__ void issue_chunk(const Params& p, uint8_t* st, uint64_t* bar,
                                            int64_t kbase, int64_t vbase, int64_t row,
                                            uint32_t rows, void* q_dst = nullptr,
                                            const void* q_src = nullptr, uint32_t q_bytes = 0) {
  using G = Geo<BITS, D, GS>;
  using Lay = StageLayout<BITS, D, GS, CH>;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_expect_tx(bar, rows * G::ROWB + (q_dst ? q_bytes : 0u));
  if (q_dst) bulk_g2s(q_dst, q_src, q_bytes, bar);
  bulk_g2s(st + Lay::O_KP, p.kp + (kbase + row) * G::KRB, rows * G::KRB, bar);
  bulk_g2s(st + Lay::O_KS, p.ks + (kbase + row) * G::NG, rows * G::SRB, bar);
  bulk_g2s(st + Lay::O_KB, p.kb + (kbase + row) * G::NG, rows * G::SRB, bar);
  bulk_g2s(st + Lay::O_VP, p.vp + (vbase + row) * G::KRB, rows * G::KRB, bar);
  bulk_g2s(st + Lay::O_VS, p.vs + (vbase + row) * G::NG, rows * G::SRB, bar);
  bulk_g2s(st + Lay::O_VB, p.vb + (vbase + row) * G::NG, rows * G::SRB, bar);
}

// Barrier among the consumer warps only (the producer warp streams on).
__device__ __forceinline__ void consumer_sync(int nthreads) { bar_sync1(nthreads); }

// ------------------------------------------------------------ split kernel --

template <int BITS, int D, int GS, int NT, int W, int RW, int STAGES, bool BF>
__global__ void __launch_bounds__((W + 1) * 32, NT == 1 ? 3 : 1) attn_kernel(const Params p) {
  using S = Smem<BITS, D, GS, NT, W, RW, STAGES>;
  constexpr int HQ = S::HQ;
  constexpr int CH = S::CH;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BARS);
  uint64_t* empty = full + STAGES;
  int* ctrl = reinterpret_cast<int*>(smem + S::CTRL);
  uint8_t* stages = smem + S::STAGES_OFF;
  float* mrg = reinterpret_cast<float*>(smem + S::STAGES_OFF);  // aliases stages after the loop
  float* wm = reinterpret_cast<float*>(smem + S::WM);
  float* wl = reinterpret_cast<float*>(smem + S::WL);
  float* rm = reinterpret_cast<float*>(smem + S::RM);
  float* rl = reinterpret_cast<float*>(smem + S::RL);
  float* sw = reinterpret_cast<float*>(smem + S::SW);
  float* sl = reinterpret_cast<float*>(smem + S::SL);
  float* ra = reinterpret_cast<float*>(smem + S::RA);

  // launched as a programmatic dependent (launch_pdl)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const bool producer = warp == W;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y % p.Hkv;
  const int qb = blockIdx.y / p.Hkv;
  const int b = blockIdx.z;
  const int nrep = p.nrep, L = p.L;
  const int qrows = nrep * L;
  const int qr0 = qb * HQ;

  int Nb = p.N;
  if (p.seq_lens) Nb = min(max(p.seq_lens[b], 0), p.N);

  // Key range of this query block (union over its rows), then this split's share.
  int lo = 0, hi = Nb;
  if (p.mask_mode == 1) {
    const int qr_last = min(qr0 + HQ, qrows) - 1;
    const int pos_first = Nb - L + qr0 / nrep, pos_last = Nb - L + qr_last / nrep;
    hi = min(Nb, pos_last + 1);
    if (p.window > 0) lo = max(0, pos_first - p.window + 1) / kTile * kTile;
    if (hi < lo) hi = lo;
  }
  const int nact = max(1, (hi - lo + p.rps - 1) / p.rps);
  if (split >= nact) return;
  const int n0 = lo + split * p.rps;
  const int n1 = min(n0 + p.rps, hi);
  const int nchunks = (n1 - n0 + CH - 1) / CH;

  if (tid == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Causal bounds shared by every column of the block (fast-path test).
  int kz_min = Nb - 1, ka_max = 0;
  if (p.mask_mode == 1) {
    const int qr_last = min(qr0 + HQ, qrows) - 1;
    kz_min = min(kz_min, Nb - L + qr0 / nrep);
    if (p.window > 0) ka_max = max(0, Nb - L + qr_last / nrep - p.window + 1);
  }
  __syncthreads();

  bool hung = false;
  const int64_t kbase = (int64_t)b * p.k_bstride + (int64_t)kvh * p.k_hstride;
  const int64_t vbase = (int64_t)b * p.v_bstride + (int64_t)kvh * p.v_hstride;
  // Producer: one chunk of CH key rows into stage c % STAGES.  Stages are
  // only reused after the `empty` barrier shows all consumers are done.
  auto produce = [&](int c) -> bool {
    const int s = c % STAGES;
    if (c >= STAGES && !mbar_wait(&empty[s], (uint32_t)(((c / STAGES) & 1) ^ 1))) return false;
    const int row = n0 + c * CH;
    const int rows = min(CH, n1 - row);
    const uint32_t cr = (uint32_t)((rows + kTile - 1) / kTile * kTile);
    issue_chunk<BITS, D, GS, CH>(p, stages + s * S::STAGE, &full[s], kbase, vbase, row, cr);
    return true;
  };
  // Prologue before any block-wide barrier: fill the ring (no waits needed).
  if (producer && lane == 0)
    for (int c = 0; c < STAGES && c < nchunks; c++) produce(c);

  WarpAcc<BITS, D, GS, NT> A;
  A.reset();

  if (producer) {
    if (lane == 0)
      for (int c = STAGES; c < nchunks; c++)
        if (!produce(c)) {
          hung = true;
          break;
        }
  } else {
    QFrag<BITS, D, GS, NT> Q;
    load_qfrag<BITS, D, GS, NT, BF>(Q, p, b, kvh, qr0, qrows, g, t);
    int klo[NT][2], khi[NT][2];
    column_bounds<NT>(klo, khi, p, qr0, qrows, Nb, t);
    for (int c = 0; c < nchunks; c++) {
      const int s = c % STAGES;
      // The decision must be warp-uniform: the slice is full of warp-collective ops.
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (uint32_t)((c / STAGES) & 1)))) {
        hung = true;
        break;
      }
      const int srow0 = n0 + c * CH + warp * RW;  // first key row of this slice
      if (srow0 < n1) {
        const bool fast = !p.scores && srow0 + RW <= n1 && srow0 + RW - 1 <= kz_min &&
                          srow0 >= ka_max;
        run_slice<BITS, D, GS, NT, RW, CH, BF>(A, Q, p, stages + s * S::STAGE, warp * RW,
                                                   srow0, n1, fast, klo, khi, qr0, qrows, kvh, b,
                                                   g, t);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (hung && lane == 0) atomicExch(p.err, 1);

  // ---- finish each consumer warp; combine the warps in shared memory ----
  warp_reduce<BITS, D, GS, NT>(A);
  if (!producer && g == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int hh = 0; hh < 2; hh++) wm[warp * HQ + nt * 8 + 2 * t + hh] = A.m_run[nt][hh];
  }
  __syncthreads();  // every stage consumed (ring reusable) and warp maxima visible
  if (!producer) {
    rescale_warp<BITS, D, GS, NT, W>(A, wm, wl, rm, warp, g, t);
    store_warp<BITS, D, GS, NT, false>(A, mrg + warp * HQ * (D + kRowPad), g, t);
  }
  __syncthreads();
  if (tid < HQ) {
    float Ls = 0.0f;
#pragma unroll
    for (int w = 0; w < W; w++) Ls += wl[w * HQ + tid];
    rl[tid] = Ls;
  }
  __syncthreads();

  // ---- combine warps; write the CTA partial or the final result ----
  const int rows_here = min(HQ, qrows - qr0);
  const int64_t cta = ((int64_t)b * p.Hkv + kvh) * p.QB + qb;
  const bool single = nact == 1;
  for (int i = tid; i < rows_here * D; i += (W + 1) * 32) {
    const int r = i / D, d = i - r * D;
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < W; w++) O += mrg[(w * HQ + r) * (D + kRowPad) + d];
    const float Lsum = rl[r], M = rm[r];
    const int qr = qr0 + r, l = qr / nrep, hq = kvh * nrep + (qr - l * nrep);
    const int64_t orow = ((int64_t)b * p.Hq + hq) * L + l;
    if (single) {
      write_row<D, BF>(p, orow, d, O, M, Lsum);
    } else {
      const int64_t slot = (cta * p.nsplit + split) * HQ + r;
      p.ws_o[slot * D + d] = O;
      if (d == 0) {
        p.ws_ml[slot * 2] = M;
        p.ws_ml[slot * 2 + 1] = Lsum;
      }
    }
  }
  if (single) return;

  // ---- last CTA of this (b, kv head, query block) merges the splits ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.counters[cta], 1u);
    ctrl[0] = (prev == (unsigned)(nact - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!ctrl[0]) return;
  __threadfence();
  merge_slots<D, HQ, (W + 1) * 32, BF>(
      p, cta * p.nsplit, nact, rows_here, sw, sl, rm, rl, ra, mrg, tid, [&](int r) -> int64_t {
        const int qr = qr0 + r, l = qr / nrep, hq = kvh * nrep + (qr - l * nrep);
        return ((int64_t)b * p.Hq + hq) * L + l;
      });
  if (tid == 0) p.counters[cta] = 0u;  // leave the ticket ready for the next call
}

// --------------------------------------------------------- balanced kernel --
//
// Decode (L = 1, no window) over one resident wave of CTAs, in two launches:
//
// attn_bal_kernel: the key tiles (16 rows) of all units u = b*Hkv + kvh are
// laid end to end, unit u owning tiles [U_u, U_u + T_u); working CTA i of C
// streams tiles [i*RT/C, (i+1)*RT/C) of the RT in total, so every CTA moves
// the same bytes whatever the lengths in the batch.  Where its range crosses
// a unit boundary it closes one segment (the part of a unit it holds) and
// opens the next.  A segment closes warp by warp, with no block barrier:
// each consumer warp writes its own partial (m, l, o) of the segment's
// query rows to partial slot (i + u)*W + warp and goes on streaming, so the
// ring never stalls at a boundary.  The holders of u are consecutive CTAs,
// so its partials fill consecutive slots.
//
// attn_bal_merge_kernel: one CTA per (unit, query row) combines the unit's
// partials (log-sum-exp, in slot order: deterministic) into the output.  It
// is launched as a programmatic dependent of the attention kernel and waits
// on its completion before reading.

// One consumer warp's partial of the live query rows (qrows): m, l per row
// and o = o_acc * fac + sum(p * bias) per (row, d), into dst = [HQ] m,
// [HQ] l, [HQ][D] o.
template <int BITS, int D, int GS, int NT>
__device__ __forceinline__ void write_warp_partial(const WarpAcc<BITS, D, GS, NT>& A, float* dst,
                                                   int qrows, int g, int t) {
  using G = Geo<BITS, D, GS>;
  constexpr int HQ = 8 * NT;
  constexpr int V = GS / 8;  // consecutive d per lane per (group, row): d = grp*GS + g*V + sl
  static_assert(V == G::C * G::E && V == 2 * G::MTG && V % 4 == 0, "lane d layout");
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int col = nt * 8 + 2 * t + hh;
      if (col >= qrows) continue;
      if (g == 0) {
        dst[col] = A.m_run[nt][hh];
        dst[HQ + col] = A.l_run[nt][hh];
      }
#pragma unroll
      for (int grp = 0; grp < G::NG; grp++) {
        float v[V];
#pragma unroll
        for (int sl = 0; sl < V; sl++) {
          const int mt = sl % G::MTG, half = sl / G::MTG;
          const float fac = (BITS == 4 && (mt & 1)) ? kCodeUnitInv * 0.0625f : kCodeUnitInv;
          v[sl] = fmaf(A.o_acc[grp * G::MTG + mt][nt][half * 2 + hh], fac, A.pb[nt][grp][hh]);
        }
        float* o = dst + 2 * HQ + col * D + grp * GS + g * V;
#pragma unroll
        for (int q4 = 0; q4 < V / 4; q4++)
          *reinterpret_cast<float4*>(o + 4 * q4) =
              make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
      }
    }
}

// Working CTAs of the balanced decode: at most one per kBalMinTiles key
// tiles and at most the launched grid, so every working CTA's range is
// non-empty and the holders of a unit are consecutive CTAs.
__device__ __forceinline__ int bal_working_ctas(int64_t RT, int grid) {
  int64_t c = RT / kBalMinTiles;
  if (c > grid) c = grid;
  if (c < 1) c = 1;
  return (int)c;
}

template <int BITS, int D, int GS, int NT, int W, int RW, int STAGES, bool BF>
__global__ void __launch_bounds__((W + 1) * 32, NT == 1 ? 3 : 1) attn_bal_kernel(const Params p) {
  using S = BalSmem<BITS, D, GS, NT, W, RW, STAGES>;
  constexpr int HQ = S::HQ;
  constexpr int CH = S::CH;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BARS);
  uint64_t* empty = full + STAGES;
  volatile int* ctrl = reinterpret_cast<volatile int*>(smem + S::CTRL);  // [1] abort
  uint64_t* qfb = reinterpret_cast<uint64_t*>(smem + S::CTRL + 8);  // second segment's fragments built
  uint8_t* stages = smem + S::STAGES_OFF;
  int* blen = reinterpret_cast<int*>(smem + S::BL);             // [B] key rows of each entry
  int64_t* bfirst = reinterpret_cast<int64_t*>(smem + S::BS);   // [B+1] first tile of each entry

  // The merge kernel may be scheduled now; it waits for this grid to finish.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const bool producer = warp == W;
  const int i = blockIdx.x;
  const int Hkv = p.Hkv, nrep = p.nrep, qrows = nrep, B = p.B;
  const bool ragged = p.seq_lens != nullptr;

  if (tid == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    mbar_init(qfb, 32);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    ctrl[1] = 0;
  }
  // Launched as a programmatic dependent (launch_pdl): each thread executes
  // griddepcontrol.wait — the previous kernel (the append, typically) is
  // complete past it — just before its first global access.  With equal
  // lengths the split and the first chunk's addresses are arithmetic on the
  // launch parameters, worked out while the previous kernel still runs.
  int64_t RT = (int64_t)B * Hkv * p.Tu;
  if (ragged) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int bb = tid; bb < B; bb += blockDim.x) blen[bb] = min(max(p.seq_lens[bb], 0), p.N);
    __syncthreads();
    if (warp == 0) {  // exclusive scan of Hkv * ceil(len / 16)
      int64_t run = 0;
      for (int base = 0; base < B; base += 32) {
        const int bb = base + lane;
        const int64_t v = bb < B ? (int64_t)Hkv * ((blen[bb] + kTile - 1) / kTile) : 0;
        int64_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        if (bb < B) bfirst[bb] = run + incl - v;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) bfirst[B] = run;
    }
    __syncthreads();
    RT = bfirst[B];
  } else {
    __syncthreads();
  }
  const int C = bal_working_ctas(RT, gridDim.x);
  const int64_t x0 = i < C ? (int64_t)i * RT / C : RT;
  const int64_t x1 = i < C ? (int64_t)(i + 1) * RT / C : RT;

  // Unit holding tile x: batch entry b, kv head kvh, first tile U, tiles T, rows n.
  auto unit_at = [&](int64_t x, int& b, int& kvh, int64_t& U, int& T, int& n) {
    if (!ragged) {
      const int64_t u = x / p.Tu;
      b = (int)(u / Hkv);
      kvh = (int)(u - (int64_t)b * Hkv);
      U = u * p.Tu;
      T = p.Tu;
      n = p.N;
    } else {
      int lo = 0, hi = B - 1;  // last entry whose first tile is <= x
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (bfirst[mid] <= x) lo = mid;
        else hi = mid - 1;
      }
      b = lo;
      n = blen[b];
      T = (n + kTile - 1) / kTile;
      kvh = (int)((x - bfirst[b]) / T);
      U = bfirst[b] + (int64_t)kvh * T;
    }
  };

  bool hung = false;
  if (producer) {
    // The whole warp walks the chunks (lane 0 issues the copies); after the
    // first chunk it loads the second segment's query halves, and once the
    // ring is first filled it turns them into fragments for the consumers.
    QRaw<BITS, D, GS, NT> qr1;
    bool q1 = false;  // raw halves of segment 1 loaded, fragments not yet built
    int c = 0, j = 0;
    for (int64_t x = x0; x < x1 && !hung; j++) {
      int b, kvh, T, n;
      int64_t U;
      unit_at(x, b, kvh, U, T, n);
      const int64_t xe = x1 < U + T ? x1 : U + T;
      const int r0 = (int)(x - U) * kTile, r1 = (int)(xe - U) * kTile;
      const int64_t kbase = (int64_t)b * p.k_bstride + (int64_t)kvh * p.k_hstride;
      const int64_t vbase = (int64_t)b * p.v_bstride + (int64_t)kvh * p.v_hstride;
      const uint16_t* qsrc = p.q + ((int64_t)b * p.Hq + (int64_t)kvh * nrep) * D;
      for (int row = r0; row < r1; row += CH, c++) {
        const int s = c % STAGES;
        // Staggered start: the rest of the ring is requested once the first
        // chunk has landed, so every CTA's first chunk (and its math) comes
        // ahead of the bulk of the initial fill.
        bool ok = !ctrl[1];
        if (ok && c == 1) ok = mbar_wait(&full[0], 0u);
        if (ok && c >= STAGES) ok = mbar_wait(&empty[s], (uint32_t)(((c / STAGES) & 1) ^ 1));
        if (!__all_sync(0xffffffffu, ok)) {
          hung = true;
          if (lane == 0) ctrl[1] = 1;
          break;
        }
        if (c == 0 && !ragged) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0)
          issue_chunk<BITS, D, GS, CH>(p, stages + s * S::STAGE, &full[s], kbase, vbase, row,
                                       (uint32_t)min(CH, r1 - row),
                                       row == r0 && j >= 2 ? smem + S::QS + s * S::QSLOT : nullptr,
                                       qsrc, (uint32_t)(nrep * D * 2));
        if (c == 0 && xe < x1) {
          int b1, kvh1, T1, n1;
          int64_t U1;
          unit_at(xe, b1, kvh1, U1, T1, n1);
          load_qraw<BITS, D, GS, NT>(qr1, p, b1, kvh1, 0, qrows, g, t);
          q1 = true;
        }
        if (q1 && c == STAGES - 1) {
          QFrag<BITS, D, GS, NT> Q1;
          qfrag_from_raw<BITS, D, GS, NT, BF>(Q1, qr1, p, t);
          store_qfrag<BITS, D, GS, NT>(Q1, smem + S::QF, lane);
          mbar_arrive(qfb);  // every lane, after its own stores
          q1 = false;
        }
      }
      x = xe;
    }
    if (q1 && !hung) {  // fewer chunks than ring stages
      QFrag<BITS, D, GS, NT> Q1;
      qfrag_from_raw<BITS, D, GS, NT, BF>(Q1, qr1, p, t);
      store_qfrag<BITS, D, GS, NT>(Q1, smem + S::QF, lane);
      mbar_arrive(qfb);
    }
  } else {
    WarpAcc<BITS, D, GS, NT> A;
    QFrag<BITS, D, GS, NT> Q;
    // Query groups: the first segment's straight from global memory into
    // every warp's registers, while the ring's first chunk is in flight;
    // the second's built by the producer warp into shared memory; later
    // segments' carried by their first chunk.
    int c = 0, j = 0;
    for (int64_t x = x0; x < x1; j++) {
      int b, kvh, T, n;
      int64_t U;
      unit_at(x, b, kvh, U, T, n);
      const int64_t xe = x1 < U + T ? x1 : U + T;
      const int r0 = (int)(x - U) * kTile, r1 = (int)(xe - U) * kTile;
      const int n1 = min(r1, n);
      int klo[NT][2], khi[NT][2];
      column_bounds<NT>(klo, khi, p, 0, qrows, n, t);
      A.reset();
      if (j == 0) {
        if (!ragged) asm volatile("griddepcontrol.wait;" ::: "memory");
        load_qfrag<BITS, D, GS, NT, BF>(Q, p, b, kvh, 0, qrows, g, t);
      } else if (j == 1) {
        const bool ok = !hung && !ctrl[1] && mbar_wait(qfb, 0u);
        if (!__all_sync(0xffffffffu, ok)) {
          if (!hung && lane == 0) ctrl[1] = 1;
          hung = true;
        }
        load_qfrag_slot<BITS, D, GS, NT>(Q, smem + S::QF, lane);
      }
      for (int row = r0; row < r1; row += CH, c++) {
        const int s = c % STAGES;
        // Warp-uniform decision: the slice is full of warp-collective ops.
        // After a timeout anywhere, skip the waits but keep the structure.
        const bool ok = !hung && !ctrl[1] && mbar_wait(&full[s], (uint32_t)((c / STAGES) & 1));
        if (!__all_sync(0xffffffffu, ok)) {
          if (!hung && lane == 0) ctrl[1] = 1;
          hung = true;
          continue;
        }
        if (row == r0 && j >= 2)  // a later segment's query group came with its first chunk
          load_qfrag<BITS, D, GS, NT, BF>(Q, p, b, kvh, 0, qrows, g, t,
                                          reinterpret_cast<const uint16_t*>(smem + S::QS +
                                                                            s * S::QSLOT));
        const int srow0 = row + warp * RW;
        if (srow0 < n1)
          run_slice<BITS, D, GS, NT, RW, CH, BF>(A, Q, p, stages + s * S::STAGE, warp * RW,
                                                     srow0, n1, srow0 + RW <= n1, klo, khi, 0,
                                                     qrows, kvh, b, g, t);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // ---- close the segment: this warp's partial, no block barrier ----
      warp_reduce<BITS, D, GS, NT>(A);
      const int64_t slot = ((int64_t)i + b * Hkv + kvh) * W + warp;
      write_warp_partial<BITS, D, GS, NT>(A, p.ws_o + slot * HQ * (D + 2), qrows, g, t);
      x = xe;
    }
  }
  if (hung && lane == 0) atomicExch(p.err, 1);
}

// Combine the partial slots of unit blockIdx.x for query row blockIdx.y,
// columns [blockIdx.z * D / DC, (blockIdx.z + 1) * D / DC); blockDim.x ==
// MG * D / DC: thread (group gi, column d).  The unit's slots are cut into
// G <= MG contiguous runs of at least 16 (one run when there are few);
// group gi folds run gi 32 (wide: 16) slots at a time — every thread loads the
// batch's (m, l) and its own o[d] in one round (coalesced across d) — into
// a running (M, L, o) in slot order, and group 0 combines the runs in run
// order (deterministic: the same sums in every thread and on every call
// with these shapes).  Long units spread over many CTAs (one long
// sequence) thus merge in one or two rounds on D / 32 blocks per row.
constexpr int kMergeSlots = 4096;  // partial slots per unit at most (launch shape)
// The wide merge: 16 slot groups of one warp each (512 threads a block),
// each lane one d of a 32-wide slice of the row, the slices spread over
// gridDim.z = D / 32 blocks, so a long unit's merge runs on D / 32 times
// more SMs and folds a sixteenth of the slots per thread.  The narrow merge
// (MG = 1, DC = 1, D threads) serves launches whose units have few slots
// each, where extra groups would sit idle.
constexpr int kWideMergeGroups = 16;
template <int D>
constexpr int wide_merge_chunks() {
  return D / 32;
}
constexpr int kWideMergeSlots = 64;  // slots per unit above which the wide merge runs
template <int D, int W, int NT, bool BF, int MG, int DC>
__global__ void __launch_bounds__(MG * (D / DC)) attn_bal_merge_kernel(const Params p, int grid) {
  constexpr int HQ = 8 * NT;
  constexpr int SLOT = HQ * (D + 2);  // floats per partial slot
  constexpr int DW = D / DC;          // d per block: one per thread of a group
  static_assert(D % DC == 0 && DW % 32 == 0, "merge slices are whole warps");
  __shared__ int64_t red_t[2];
  __shared__ float run_ml[MG][2];
  __shared__ float run_o[MG][DW];
  const int u = blockIdx.x, r = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  const int gi = tid / DW, dl = tid - gi * DW, d = blockIdx.z * DW + dl;
  const int Hkv = p.Hkv, b = u / Hkv, kvh = u - b * Hkv;
  const int64_t orow = (int64_t)b * p.Hq + kvh * p.nrep + r;

  // The unit's tiles and the partition of the attention launch.
  int64_t U, RT;
  int T;
  if (p.seq_lens == nullptr) {
    T = p.Tu;
    U = (int64_t)u * p.Tu;
    RT = (int64_t)p.B * Hkv * p.Tu;
  } else {  // tiles of the entries before b and of all entries
    // The lengths live in memory that an earlier kernel of the stream may
    // have just written (a ragged append advances them): wait before
    // reading.  The attention grid signals its dependents at its start, so
    // without this wait the merge could run ahead of the append.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    int64_t before = 0, all = 0;
    for (int bb = tid; bb < p.B; bb += blockDim.x) {
      const int n = min(max(p.seq_lens[bb], 0), p.N);
      const int64_t tb = (int64_t)Hkv * ((n + kTile - 1) / kTile);
      all += tb;
      if (bb < b) before += tb;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      all += __shfl_xor_sync(0xffffffffu, all, o);
    }
    if (tid == 0) red_t[0] = red_t[1] = 0;
    __syncthreads();
    if (lane == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&red_t[0]), (unsigned long long)before);
      atomicAdd(reinterpret_cast<unsigned long long*>(&red_t[1]), (unsigned long long)all);
    }
    __syncthreads();
    const int n = min(max(p.seq_lens[b], 0), p.N);
    T = (n + kTile - 1) / kTile;
    U = red_t[0] + (int64_t)kvh * T;
    RT = red_t[1];
  }

  // Everything below reads what the attention grid wrote.  (The next
  // kernel on the stream may be scheduled meanwhile; it waits likewise.)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (T == 0) {  // an entry with no keys: a zero row (or an empty partial)
    if (gi == 0) write_row<D, BF>(p, orow, d, 0.0f, kNeg, 0.0f);
    return;
  }
  const int C = bal_working_ctas(RT, grid);
  const int i_first = (int)(((U + 1) * C - 1) / RT);
  const int i_last = (int)(((U + T) * C - 1) / RT);
  const int nslots = (i_last - i_first + 1) * W;  // <= kMergeSlots (host launch shape)
  const int G = min(MG, (nslots + 15) / 16);  // groups of at least 16 slots
  const float* base = p.ws_o + ((int64_t)i_first + u) * W * SLOT;

  float M = kNeg, L = 0.0f, acc = 0.0f;
  if (gi < G) {
    const int s0 = (int)((int64_t)gi * nslots / G), s1 = (int)((int64_t)(gi + 1) * nslots / G);
    // slots per round: 32 in the narrow merge, 16 in the wide one (whose
    // groups hold about 16 slots each, within 128 registers a thread)
    constexpr int NB = MG > 1 ? 16 : 32;
    for (int j0 = s0; j0 < s1; j0 += NB) {
      const int nj = min(NB, s1 - j0);
      float m[NB], l[NB], o[NB];
#pragma unroll
      for (int k = 0; k < NB; k++) {
        const bool v = k < nj;
        const float* sp = base + (int64_t)(j0 + k) * SLOT;
        m[k] = v ? __ldcg(sp + r) : kNeg;
        l[k] = v ? __ldcg(sp + HQ + r) : 0.0f;
        o[k] = v ? __ldcg(sp + 2 * HQ + r * D + d) : 0.0f;
      }
      float Mn = M;
#pragma unroll
      for (int k = 0; k < NB; k++) Mn = fmaxf(Mn, m[k]);
      const float a = ex2((M - Mn) * kLog2e);
      L *= a;
      acc *= a;
#pragma unroll
      for (int k = 0; k < NB; k++) {
        const float w = ex2((m[k] - Mn) * kLog2e);
        L = fmaf(l[k], w, L);
        acc = fmaf(o[k], w, acc);
      }
      M = Mn;
    }
  }
  if (G == 1) {
    if (gi == 0) write_row<D, BF>(p, orow, d, acc, M, L);
    return;
  }
  if (gi < G) {
    run_o[gi][dl] = acc;
    if (dl == 0) {
      run_ml[gi][0] = M;
      run_ml[gi][1] = L;
    }
  }
  __syncthreads();
  if (gi == 0) {
    float Mt = kNeg;
    for (int k = 0; k < G; k++) Mt = fmaxf(Mt, run_ml[k][0]);
    float Lt = 0.0f, At = 0.0f;
    for (int k = 0; k < G; k++) {
      const float w = ex2((run_ml[k][0] - Mt) * kLog2e);
      Lt = fmaf(run_ml[k][1], w, Lt);
      At = fmaf(run_o[k][dl], w, At);
    }
    write_row<D, BF>(p, orow, d, At, Mt, Lt);
  }
}

// ------------------------------------------------------------ host side --

constexpr int kWarps = 4;  // consumer warps per CTA (+1 producer)

// Rows per consumer slice: 32 when registers allow, else 16.
template <int D, int NT>
constexpr int rows_per_warp() {
  return (D * NT <= 128) ? 32 : 16;
}

template <int BITS, int D, int GS, int RW>
constexpr int stages_for() {
  constexpr int stage = kWarps * RW * Geo<BITS, D, GS>::ROWB;
  return stage <= 12 * 1024 ? 4 : (stage <= 24 * 1024 ? 3 : 2);
}

struct LaunchShape {
  int QB, nsplit, rps;
  int ctas = 0;        // > 0: balanced kernel with this many CTAs (one wave)
  bool small = false;  // balanced kernel with 16-row slices (short per-CTA ranges)
};

// Balanced decode: at most this many key rows per CTA take the 16-row-slice
// instance (64-row chunks, 4 ring stages): its first chunk lands sooner and
// a short range still fills the ring; longer ranges are issue-bound and
// take the 32-row slices.
constexpr int kBalSmallRows = 448;

inline int num_sms(int dev) {
  static int g_num_sms[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!g_num_sms[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    g_num_sms[dev] = v;
  }
  return g_num_sms[dev];
}

// Key split: one resident wave of CTAs (SM count x blocks per SM of this
// kernel); each split a multiple of 16 key rows (the TMA row unit) and at
// most kMergeMax splits per merge group.
inline LaunchShape shape_for(int B, int Hkv, int nrep, int L, int N, int NT, int target_ctas) {
  LaunchShape s;
  const int HQ = 8 * NT;
  s.QB = (nrep * L + HQ - 1) / HQ;
  const int64_t units = (int64_t)B * Hkv * s.QB;
  // round down: one CTA too many would start a second wave for itself
  int nsplit = (int)std::max<int64_t>(1, target_ctas / units);
  const int min_rows = 256;
  nsplit = std::min(nsplit, std::max(1, (N + min_rows - 1) / min_rows));
  nsplit = std::min(nsplit, kMergeMax);
  int rps = (N + nsplit - 1) / nsplit;
  rps = (rps + kTile - 1) / kTile * kTile;
  if (rps <= 0) rps = kTile;
  s.rps = rps;
  s.nsplit = std::max(1, (N + rps - 1) / rps);
  return s;
}

// Workspace layout (fixed prefix, so every call finds its tickets at the
// same place whatever the previous call's shape was):
//   [0, 256)                      device error flag
//   [256, 256 + 4*kMaxTickets)    split tickets, zero between calls
//   then (m, l) and o partials of the splits.
constexpr int64_t kMaxTickets = 65536;
constexpr size_t kTicketOff = kWsFlagBytes;
constexpr size_t kPartialOff = kTicketOff + 4 * kMaxTickets;

// Balanced decode partials: (ctas + units) groups of kWarps slots of
// [HQ] m, [HQ] l, [HQ][D] o floats.
inline size_t bal_group_bytes(int NT, int D) { return (size_t)kWarps * 8 * NT * (D + 2) * 4; }
inline size_t bal_slot_groups(int ctas, int B, int Hkv) { return (size_t)ctas + (size_t)B * Hkv; }

inline size_t ws_bytes_for(int B, int Hkv, const LaunchShape& s, int NT, int D) {
  if (s.ctas > 0)  // balanced: one (m, l, o) partial per warp, slots (i + u) * W + warp
    return kPartialOff + bal_slot_groups(s.ctas, B, Hkv) * bal_group_bytes(NT, D);
  if (s.nsplit <= 1) return kPartialOff;
  const size_t slots = (size_t)B * Hkv * s.QB * s.nsplit * 8 * NT;
  return kPartialOff + (slots * 2 * 4 + 255) / 256 * 256 + slots * D * 4;
}

// Launch one kernel instance: the balanced decode kernel when s.ctas > 0,
// else the split kernel.  Blocks per SM are queried once per (kernel,
// device) and cached (kernel_setup).
template <int BITS, int D, int GS, int NT, int RW>
int32_t launch_rw(Params& p, const LaunchShape& s, int B, cudaStream_t st, int* occ) {
  constexpr int ST = stages_for<BITS, D, GS, RW>();
  const bool bal = s.ctas > 0;
  const int smem = bal ? BalSmem<BITS, D, GS, NT, kWarps, RW, ST>::TOTAL
                       : Smem<BITS, D, GS, NT, kWarps, RW, ST>::TOTAL;
  void (*kern)(Params);
  if (bal)
    kern = p.bf16 ? attn_bal_kernel<BITS, D, GS, NT, kWarps, RW, ST, true>
                  : attn_bal_kernel<BITS, D, GS, NT, kWarps, RW, ST, false>;
  else
    kern = p.bf16 ? attn_kernel<BITS, D, GS, NT, kWarps, RW, ST, true>
                  : attn_kernel<BITS, D, GS, NT, kWarps, RW, ST, false>;
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  int nb = 1;
  int32_t rc = kernel_setup(reinterpret_cast<const void*>(kern), (kWarps + 1) * 32, smem, dev, &nb);
  if (rc) return rc;
  if (occ) {
    *occ = nb;
    return KVQ_OK;
  }
  const dim3 grid = bal ? dim3(s.ctas) : dim3(s.nsplit, p.Hkv * s.QB, B);
  KVQ_CUDA_TRY(launch_pdl(kern, grid, dim3((kWarps + 1) * 32), (size_t)smem, st, p));
  if (bal) {
    // merge of the per-warp partials, a programmatic dependent of the
    // attention grid (it waits for that grid inside, with griddepcontrol)
    // (wide when the units have many slots each: one long sequence)
    constexpr int MG = kWideMergeGroups, DC = wide_merge_chunks<D>();
    const bool wide = (int64_t)s.ctas * kWarps > (int64_t)kWideMergeSlots * B * p.Hkv;
    void (*merge)(Params, int) =
        wide ? (p.bf16 ? attn_bal_merge_kernel<D, kWarps, NT, true, MG, DC>
                       : attn_bal_merge_kernel<D, kWarps, NT, false, MG, DC>)
             : (p.bf16 ? attn_bal_merge_kernel<D, kWarps, NT, true, 1, 1>
                       : attn_bal_merge_kernel<D, kWarps, NT, false, 1, 1>);
    KVQ_CUDA_TRY(launch_pdl(merge, dim3((unsigned)(B * p.Hkv), (unsigned)p.nrep, wide ? DC : 1),
                            dim3(wide ? MG * (D / DC) : D), 0, st, p, s.ctas));
  }
  return KVQ_OK;
}

template <int BITS, int D, int GS, int NT>
int32_t launch_t(Params& p, const LaunchShape& s, int B, cudaStream_t st, int* occ) {
  constexpr int RW = rows_per_warp<D, NT>();
  if constexpr (RW == 32) {
    if (s.ctas > 0 && s.small) return launch_rw<BITS, D, GS, NT, 16>(p, s, B, st, occ);
  }
  return launch_rw<BITS, D, GS, NT, RW>(p, s, B, st, occ);
}

template <int BITS, int D, int GS>
int32_t pick_nt(Params& p, const LaunchShape& s, int NT, int B, cudaStream_t st, int* occ) {
  if (NT == 1) return launch_t<BITS, D, GS, 1>(p, s, B, st, occ);
  return launch_t<BITS, D, GS, 2>(p, s, B, st, occ);
}

template <int BITS, int D>
int32_t pick_gs(Params& p, const LaunchShape& s, int GSv, int NT, int B, cudaStream_t st, int* occ) {
  switch (GSv) {
    case 32: return pick_nt<BITS, D, 32>(p, s, NT, B, st, occ);
    case 64: return pick_nt<BITS, D, 64>(p, s, NT, B, st, occ);
    case 128:
      if constexpr (D >= 128) return pick_nt<BITS, D, 128>(p, s, NT, B, st, occ);
      break;
  }
  return fail(KVQ_ERR_ARG, "attention: unsupported group_size for this head_dim");
}

template <int BITS>
int32_t pick_d(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st,
               int* occ) {
  switch (Dv) {
    case 64: return pick_gs<BITS, 64>(p, s, GSv, NT, B, st, occ);
    case 128: return pick_gs<BITS, 128>(p, s, GSv, NT, B, st, occ);
    case 256: return pick_gs<BITS, 256>(p, s, GSv, NT, B, st, occ);
  }
  return fail(KVQ_ERR_ARG, "attention: head_dim must be 64, 128 or 256");
}

// The tcgen05 chunked prefill (kvq_prefill_tc.cu): 8-bit codes, D 128, group 64.
bool prefill_tc_supported(int bits, int D, int gs, int L, bool scores);
int32_t launch_prefill_tc(Params& p, int B, void* ws, size_t ws_bytes, cudaStream_t st);
// The warp-specialised tcgen05 prefill (kvq_prefill_tc2.cu): fp16 caches,
// D 128, 4- or 8-bit codes, group 32 / 64 / 128.
bool prefill_tc2_supported(int bits, int D, int gs, int dtype, int L);
int32_t launch_prefill_tc2(Params& p, int B, int bits, int gs, void* ws, size_t ws_bytes,
                           cudaStream_t st);

// Per-width launchers (one translation unit each, compiled in parallel);
// s.ctas > 0 selects the balanced kernel.  With occ != nullptr they only
// report that kernel's resident blocks per SM.
int32_t dispatch_b4(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st, int* occ);
int32_t dispatch_b8(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st, int* occ);

}  // namespace attn
}  // namespace kvq
