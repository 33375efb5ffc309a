#pragma once
// kvq_tc.cuh — pieces shared by the two tcgen05 chunked-prefill kernels
// (kvq_prefill_tc.cu, kvq_prefill_tc2.cu): 128-byte-swizzled shared-memory
// tiles and their UMMA descriptors, the tcgen05 MMA / TMEM wrappers, the
// balanced-grid partition of the key tiles of all units, and the merge of
// units cut between CTAs.
#include "kvq_attn_impl.cuh"

namespace kvq {
namespace attn {
namespace tc {

constexpr int kRows = 128;  // query rows per unit (TMEM lanes)
constexpr int TD = 128;     // head dim of the tensor-core prefill kernels
// One partial row of the balanced grid: m, l, sum(p vb_0), sum(p vb_1), O'[128]
constexpr int kSlotRow = 4 + TD;

// byte offset of element (row, c) of a 128-byte-swizzled tile of 64-element rows
__device__ __forceinline__ uint32_t sw128(int row, int c) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + (((c >> 3) ^ (row & 7)) << 4) + (c & 7) * 2);
}

// UMMA shared-memory descriptor: 128-byte swizzle, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// instruction descriptor, kind::f16: f16 A/B, f32 accumulate
__device__ __forceinline__ uint32_t idesc_f16(int M, int N, int b_mn_major) {
  return (1u << 4) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}

__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
        "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
        "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(addr));
}

__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Key range [lo, hi) of query block qt (the union over its rows; lo tile
// aligned) and its count of KT-key tiles.  Host and device use the same
// rule, so the host can size the balanced grid.
template <int KT>
__host__ __device__ inline int tc_block_tiles(int qt, int Nb, int L, int nrep, int mask_mode,
                                              int window, int* lo_out = nullptr,
                                              int* hi_out = nullptr) {
  const int qrows = nrep * L, qr0 = qt * kRows;
  const int qr_last = (qr0 + kRows < qrows ? qr0 + kRows : qrows) - 1;
  int lo = 0, hi = Nb;
  if (mask_mode == 1) {
    const int h = Nb - L + qr_last / nrep + 1;
    hi = h < Nb ? h : Nb;
    if (window > 0) {
      const int w = Nb - L + qr0 / nrep - window + 1;
      lo = (w > 0 ? w : 0) / kTile * kTile;
    }
    if (hi < lo) hi = lo;
  }
  if (lo_out) {
    *lo_out = lo;
    *hi_out = hi;
  }
  return (hi - lo + KT - 1) / KT;
}

// Query block qt holding tile `rem` of one (b, kv head) pair's concatenated
// tile list, and the tile's index j0 inside that block: a warp-wide scan of
// the blocks' tile counts, 32 blocks per step.  All 32 lanes call it.
template <int KT>
__device__ __forceinline__ void tc_locate(int rem, int nqb, int Nb, int L, int nrep, int mask_mode,
                                          int window, int lane, int& qt, int& j0) {
  int base = 0;
  qt = nqb;
  j0 = 0;
  for (int q0 = 0; q0 < nqb; q0 += 32) {
    const int q = q0 + lane;
    const int n = q < nqb ? tc_block_tiles<KT>(q, Nb, L, nrep, mask_mode, window) : 0;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const unsigned hit =
        __ballot_sync(0xffffffffu, n > 0 && rem >= base + incl - n && rem < base + incl);
    const int src = hit ? __ffs(hit) - 1 : 0;
    const int excl = __shfl_sync(0xffffffffu, incl - n, src);
    if (hit) {
      qt = q0 + src;
      j0 = rem - base - excl;
      return;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
}

// Merge for the balanced grid: block c finishes the unit holding the first
// tile of its run when that unit began in an earlier CTA and ends within
// this run (every split unit has exactly one such CTA).  Its pieces sit in
// slot 2c' of every CTA c' after the first one (their first unit) and in
// slot 2c' + 1 of the first CTA when the unit is not where that CTA's run
// starts (its last unit).  Thread (qc, r) merges 32 columns (quarter qc) of
// row r.
constexpr int kMergeThreads = 4 * kRows;

template <bool BF, int KT>
__global__ void __launch_bounds__(kMergeThreads) prefill_tc_merge_kernel(const Params p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, r = tid & (kRows - 1), qc = tid >> 7;
  const int kh = qc >> 1;  // quantisation group of these columns
  const int nrep = p.nrep, L = p.L, qrows = nrep * L;
  const int nqb = (qrows + kRows - 1) / kRows;
  const int64_t C = p.QB;
  const int64_t T = (int64_t)p.B * p.Hkv * p.Tu;
  const int64_t c = blockIdx.x;
  const int64_t T0 = c * T / C, T1 = (c + 1) * T / C;
  const int64_t hp = T0 / p.Tu;
  int qt, jl;
  tc_locate<KT>((int)(T0 - hp * p.Tu), nqb, p.N, L, nrep, p.mask_mode, p.window, lane, qt, jl);
  const int ntl = tc_block_tiles<KT>(qt, p.N, L, nrep, p.mask_mode, p.window);
  const int64_t u0 = T0 - jl;  // first tile (in the list) of the unit holding T0
  if (u0 >= T0 || u0 + ntl > T1) return;  // starts in this run, or goes on past it
  int64_t cf = u0 * C / T;  // the CTA whose run holds u0
  while (cf + 1 < C && (cf + 1) * T / C <= u0) cf++;
  while (cf > 0 && cf * T / C > u0) cf--;
  const int qr = qt * kRows + r;
  if (qr >= qrows) return;
  const int np = (int)(c - cf + 1);  // pieces
  // piece i's row: slot 2(cf + i), or 2cf + 1 for a first piece that is not
  // where its CTA's run starts
  const size_t row0 = ((size_t)(2 * cf + (u0 > cf * T / C ? 1 : 0)) * kRows + r) * kSlotRow;
  auto piece = [&](int i) -> const float* {
    return p.ws_o + (i == 0 ? row0 : ((size_t)(2 * (cf + i)) * kRows + r) * kSlotRow);
  };
  float mx = kNeg;
  for (int i0 = 0; i0 < np; i0 += 4) {
    float mv[4];
#pragma unroll
    for (int i = 0; i < 4; i++) mv[i] = i0 + i < np ? piece(i0 + i)[0] : kNeg;
#pragma unroll
    for (int i = 0; i < 4; i++) mx = fmaxf(mx, mv[i]);
  }
  float lt = 0.0f, pb = 0.0f, o[32];
#pragma unroll
  for (int k = 0; k < 32; k++) o[k] = 0.0f;
#pragma unroll 2
  for (int i = 0; i < np; i++) {
    const float* srow = piece(i);
    const float w = ex2((srow[0] - mx) * kLog2e);
    lt = fmaf(w, srow[1], lt);
    pb = fmaf(w, srow[2 + kh], pb);
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
      const float4 v = *reinterpret_cast<const float4*>(srow + 4 + qc * 32 + k);
      o[k] = fmaf(w, v.x, o[k]);
      o[k + 1] = fmaf(w, v.y, o[k + 1]);
      o[k + 2] = fmaf(w, v.z, o[k + 2]);
      o[k + 3] = fmaf(w, v.w, o[k + 3]);
    }
  }
  const int b = (int)(hp / p.Hkv), kvh = (int)(hp - (int64_t)b * p.Hkv);
  const int l = qr / nrep, hh = qr - l * nrep;
  uint16_t* dst = p.out + (((int64_t)b * p.Hq + kvh * nrep + hh) * L + l) * TD + qc * 32;
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float v0 = lt > 0.0f ? (o[k + 2 * u] + pb) / lt : 0.0f;
      const float v1 = lt > 0.0f ? (o[k + 2 * u + 1] + pb) / lt : 0.0f;
      w[u] = (uint32_t)f_to_dt<BF>(v0) | ((uint32_t)f_to_dt<BF>(v1) << 16);
    }
    *reinterpret_cast<uint4*>(dst + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace tc
}  // namespace attn
}  // namespace kvq
