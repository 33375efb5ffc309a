// kvq_prefill_tc2.cu — warp-specialised chunked prefill on the tcgen05 tensor
// cores for fp16 caches with D = 128: 4- or 8-bit codes, group 32, 64 or 128.
//
// A unit is 128 query rows of one (batch, kv head) (TMEM lanes; rows are the
// (position, head) pairs of the GQA group), as in kvq_prefill_tc.cu.  What
// differs is where the dequantisation goes and how the warps are split:
//
//   * 6 dequantisation warps turn each 64-key tile of the TMA ring into fp16
//     operands in shared memory, K and V at the same time.  K (4 warps):
//     w = s*c + b in f32 (exact product), split into w_hi = fp16(w) and
//     w_lo = fp16(w - w_hi), so Q . w = Q . w_hi + Q . w_lo to ~22 bits — one
//     accumulator holds the whole logit (scale and bias included).  V (2
//     warps): fp16(s*c + b) with one HFMA2 per pair of codes (a code c taken
//     exactly as the fp16 1024 + c minus 1024).  A key past the valid range
//     gets zeros.
//   * 1 MMA warp (one lane issues): S_t = Q K_hi^T + Q K_lo^T (M 128, N 64,
//     K 256: 16 UMMAs) into TMEM buffer t % 3, up to two tiles ahead of
//     O += P_t V_t (M 128, N 64 per d panel, K 64; P from TMEM).
//     Completion goes to mbarriers through tcgen05.commit.
//   * 8 softmax warps, two threads per query row (warps w and w + 4 reach
//     the same TMEM lanes; each takes 32 of the tile's 64 keys): S from TMEM
//     to registers, rounded to the dtype (the reference's rounding point),
//     masked, tile maximum exchanged with the partner, lazy rescale of O
//     (only when the maximum grows by more than 2^8), p = 2^((x - m) log2 e)
//     packed to fp16 into the S buffer's first 32 columns (P aliases S), and
//     l accumulated in registers.
//   * 1 producer warp streams the six K/V arrays of each tile with 1-D bulk
//     copies into a 4-stage ring (a copy takes ~2.4 us to land; with two
//     stages the ring, not the math, set the pace).
// So the dequantisation of tile t + 1, the QK^T of tile t + 1 and the PV of
// tile t - 1 all run while the softmax warps work on tile t.
//
// Shared memory (1024-byte aligned): Q [2 d panels] SW128 [128][64] fp16;
// K [2 buffers][hi, lo][2 panels] SW128 [64][64]; V [2 buffers][2 panels]
// SW128 [64][64] (the MN-major B operand of PV); the raw ring; row exchange;
// mbarriers.  TMEM (512 columns): S buffers at 0, 64, 128; O at [256, 384).
//
// Grid and partials as in kvq_prefill_tc.cu (balanced: one CTA per SM over
// equal runs of all units' key tiles, units cut between CTAs finished by
// prefill_tc_merge_kernel; the partial rows carry O itself and zero bias
// sums).  Every wait is bounded; on timeout the kernel raises the error
// flag, and every role leaves its loop.
#include "kvq_tc.cuh"

namespace kvq {
namespace attn {
namespace {

using namespace tc;

constexpr int kKT = 64;                 // keys per tile
constexpr int kSBuf = 3;                // S buffers in TMEM
constexpr int kRaw2 = 4;                // raw ring stages (a bulk copy takes ~2.4 us to land)
constexpr int kSmWarps = 8;             // softmax warps, two per query row
constexpr int kKWarps = 4;              // K dequantisation warps
constexpr int kVWarps = 2;              // V dequantisation warps
constexpr int kCvWarps = kKWarps + kVWarps;
constexpr int kThreads2 = 16 * 32;      // 512
// Warps are spread over the SM's four sub-partitions by warp id % 4.  Each
// sub-partition holds two softmax warps (w and w + 4 reach TMEM lanes
// 32 (w % 4)); the dequantisation warps fill sub-partitions 0-2, so the MMA
// warp shares sub-partition 3 only with its two softmax warps and the
// (mostly waiting) producer: the MMA issue path is the pipeline's pace.
constexpr int kProdWarp = 11;
constexpr int kMmaWarp = 15;
__device__ __forceinline__ int k_warp_index(int w) {  // 8, 9, 10, 12 -> 0..3, else -1
  return w >= 8 && w <= 10 ? w - 8 : (w == 12 ? 3 : -1);
}
__device__ __forceinline__ int v_warp_index(int w) {  // 13, 14 -> 0..1, else -1
  return w == 13 || w == 14 ? w - 13 : -1;
}
constexpr uint32_t kTmO = 256;          // O columns [256, 384): d panel p at 256 + 64 p
constexpr int kPanelQ = kRows * 128;    // bytes of one [128][64] fp16 panel
constexpr int kPanelK = kKT * 128;      // bytes of one [64][64] fp16 panel

template <int BITS, int GS>
struct Lay2 {
  using Raw = StageLayout<BITS, TD, GS, kKT>;
  static constexpr int Q = 0;
  static constexpr int KBUF = 2 * 2 * kPanelK;  // hi, lo x 2 panels
  static constexpr int K = Q + 2 * kPanelQ;
  static constexpr int VBUF = 2 * kPanelK;
  static constexpr int V = K + 2 * KBUF;
  static constexpr int RAW = V + 2 * VBUF;
  static constexpr int XCH = RAW + kRaw2 * Raw::STAGE;  // f32 [2 parity][2 halves][128] + l [2][128]
  static constexpr int BAR = XCH + (2 * 2 + 2) * kRows * 4;
  // mbarriers: raw_full[R] raw_empty[R] k_ready[2] k_free[2] v_ready[2] v_free[2]
  //            s_full[3] p_ready[3] pv_done[3] q_ready o_free mma_end
  static constexpr int NBAR = 2 * kRaw2 + 4 * 2 + 3 * kSBuf + 3;
  static constexpr int CTL = BAR + NBAR * 8;  // TMEM base (u32), abort flag (int)
  static constexpr int TOTAL = CTL + 16 + 1024;
  static_assert(TOTAL <= 227 * 1024, "prefill tile buffers exceed the shared memory of a CTA");
  static_assert(Raw::STAGE % 16 == 0, "ring stages must stay 16-byte aligned");
};

struct Bars {
  uint64_t *raw_full, *raw_empty, *k_ready, *k_free, *v_ready, *v_free, *s_full, *p_ready,
      *pv_done, *q_ready, *o_free, *mma_end;
};

__device__ __forceinline__ Bars bars_at(uint8_t* base) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  Bars r;
  r.raw_full = b;
  r.raw_empty = b + kRaw2;
  b += 2 * kRaw2;
  r.k_ready = b;
  r.k_free = b + 2;
  r.v_ready = b + 4;
  r.v_free = b + 6;
  r.s_full = b + 8;
  r.p_ready = b + 8 + kSBuf;
  r.pv_done = b + 8 + 2 * kSBuf;
  r.q_ready = b + 8 + 3 * kSBuf;
  r.o_free = r.q_ready + 1;
  r.mma_end = r.q_ready + 2;
  return r;
}

// The CTA's units with key tiles, in order: unit (pair hp = b * Hkv + kv
// head, query block qt), its tiles [sj, j1) and key range [lo, hi).  Every
// role walks the same sequence.
struct Walk {
  int64_t t, T1, hp;
  int qt, sj, nqb, Nb;
  bool first;
  // current unit
  int j1, lo, hi, ntl;
  __device__ __forceinline__ bool next(const Params& p) {
    while (first || t < T1) {
      first = false;
      ntl = tc_block_tiles<kKT>(qt, Nb, p.L, p.nrep, p.mask_mode, p.window, &lo, &hi);
      j1 = (int)min((int64_t)ntl, (int64_t)sj + (T1 - t));
      if (j1 > sj) return true;
      advance();
    }
    return false;
  }
  __device__ __forceinline__ void advance() {
    t += j1 - sj;
    sj = 0;
    if (++qt == nqb) {
      qt = 0;
      ++hp;
    }
  }
};

// Named barrier of the two softmax warps that share query rows, which also
// ANDs their status: both see the same answer, so they leave their loops
// together and neither waits at a barrier the other no longer reaches.
__device__ __forceinline__ bool pair_and(int id, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, %2, 64, q;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id)
      : "memory");
  return r != 0;
}

// 8 consecutive codes (d0 .. d0 + 7) of a packed key row as exact floats.
template <int BITS>
__device__ __forceinline__ void load_codes8(const uint8_t* row, int d0, float (&c)[8]) {
  if constexpr (BITS == 8) {
    const uint2 w = *reinterpret_cast<const uint2*>(row + d0);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      c[i] = __uint_as_float(prmt(w.x, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
      c[4 + i] = __uint_as_float(prmt(w.y, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
    }
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + d0 / 2);
#pragma unroll
    for (int i = 0; i < 8; i++)
      c[i] = __uint_as_float(((w >> (4 * i)) & 0xFu) | 0x4B000000u) - 8388608.0f;
  }
}

template <int BITS, int GS>
__global__ void __launch_bounds__(kThreads2, 1) prefill_tc2_kernel(const Params p) {
  using LY = Lay2<BITS, GS>;
  using Raw = typename LY::Raw;
  using G = Geo<BITS, TD, GS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const Bars bar = bars_at(sm + LY::BAR);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sm + LY::CTL);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + LY::CTL + 4);
  float* xch = reinterpret_cast<float*>(sm + LY::XCH);  // [2 parity][2 halves][128]
  float* xl = xch + 4 * kRows;                          // [2 halves][128]

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nrep = p.nrep, L = p.L, qrows = nrep * L;
  Walk wk;
  wk.nqb = (qrows + kRows - 1) / kRows;
  wk.Nb = p.N;
  wk.first = true;
  if (p.QB > 0) {  // balanced grid: an equal run of all units' tiles
    const int64_t T = (int64_t)p.B * p.Hkv * p.Tu;
    const int64_t T0 = (int64_t)blockIdx.x * T / p.QB;
    wk.T1 = (int64_t)(blockIdx.x + 1) * T / p.QB;
    wk.t = T0;
    wk.hp = T0 / p.Tu;
    tc_locate<kKT>((int)(T0 - wk.hp * p.Tu), wk.nqb, wk.Nb, L, nrep, p.mask_mode, p.window,
                   lane, wk.qt, wk.sj);
  } else {  // one CTA per unit: (query block, kv head, b)
    wk.hp = (int64_t)blockIdx.z * p.Hkv + blockIdx.y;
    wk.qt = blockIdx.x;
    wk.sj = 0;
    wk.t = 0;
    wk.T1 = tc_block_tiles<kKT>(wk.qt, wk.Nb, L, nrep, p.mask_mode, p.window);
    wk.nqb = wk.qt + 1;  // never walks past its unit
    if (p.seq_lens) wk.Nb = min(max(p.seq_lens[blockIdx.z], 0), p.N);
  }

  if (tid == 0) {
    for (int s = 0; s < kRaw2; s++) {
      mbar_init(&bar.raw_full[s], 1);
      mbar_init(&bar.raw_empty[s], kCvWarps);  // K and V warps release a stage
    }
    for (int s = 0; s < 2; s++) {
      mbar_init(&bar.k_ready[s], kKWarps);
      mbar_init(&bar.k_free[s], 1);
      mbar_init(&bar.v_ready[s], kVWarps);
      mbar_init(&bar.v_free[s], 1);
    }
    for (int s = 0; s < kSBuf; s++) {
      mbar_init(&bar.s_full[s], 1);
      mbar_init(&bar.p_ready[s], kSmWarps);
      mbar_init(&bar.pv_done[s], 1);
    }
    mbar_init(bar.q_ready, kSmWarps);
    mbar_init(bar.o_free, kSmWarps);
    mbar_init(bar.mma_end, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tmem_holder;
  bool hung = false;
  // warp-uniform bounded wait: false (and the abort flag) on timeout or abort
  auto wait_all = [&](uint64_t* b, uint32_t parity) -> bool {
    const bool ok = !hung && !*abort_flag && mbar_wait(b, parity);
    if (!__all_sync(0xffffffffu, ok)) {
      if (!hung && lane == 0) *abort_flag = 1;
      hung = true;
      return false;
    }
    return true;
  };

  if (warp == kProdWarp) {
    // ---------------- producer: the raw ring ----------------
    int tc = 0;
    while (!hung && wk.next(p)) {
      const int b = (int)(wk.hp / p.Hkv), kvh = (int)(wk.hp - (int64_t)b * p.Hkv);
      const int64_t kbase = (int64_t)b * p.k_bstride + (int64_t)kvh * p.k_hstride;
      const int64_t vbase = (int64_t)b * p.v_bstride + (int64_t)kvh * p.v_hstride;
      for (int j = wk.sj; j < wk.j1; j++, tc++) {
        const int s = tc % kRaw2;
        if (tc >= kRaw2 && !wait_all(&bar.raw_empty[s], (uint32_t)(((tc / kRaw2) & 1) ^ 1))) break;
        const int row = wk.lo + j * kKT;
        const int rows = min(kKT, wk.hi - row);
        if (lane == 0)
          issue_chunk<BITS, TD, GS, kKT>(p, sm + LY::RAW + s * Raw::STAGE, &bar.raw_full[s],
                                          kbase, vbase, row,
                                          (uint32_t)((rows + kTile - 1) / kTile * kTile));
      }
      wk.advance();
    }
    // copies issued and never consumed (abort) must land before the CTA exits
    for (int k = max(0, tc - kRaw2); k < tc; k++)
      if (lane == 0) mbar_wait(&bar.raw_full[k % kRaw2], (uint32_t)((k / kRaw2) & 1));
  } else if (k_warp_index(warp) >= 0) {
    // ---------------- K dequantisation: w = s*c + b -> fp16 hi + lo ----------------
    const int ct = k_warp_index(warp) * 32 + lane;
    constexpr int kKThreads = kKWarps * 32;
    int tc = 0;
    while (!hung && wk.next(p)) {
      for (int j = wk.sj; j < wk.j1 && !hung; j++, tc++) {
        const int s = tc % kRaw2, buf = tc & 1;
        const int n0 = wk.lo + j * kKT;
        const uint8_t* st = sm + LY::RAW + s * Raw::STAGE;
        if (!wait_all(&bar.raw_full[s], (uint32_t)((tc / kRaw2) & 1))) break;
        if (tc >= 2 && !wait_all(&bar.k_free[buf], (uint32_t)(((tc >> 1) & 1) ^ 1))) break;
        uint8_t* khi = sm + LY::K + buf * LY::KBUF;
        uint8_t* klo = khi + 2 * kPanelK;
        // job: (key, 8 consecutive d); 64 keys x 16 chunks
#pragma unroll 2
        for (int it = 0; it < (kKT * 16) / kKThreads; it++) {
          const int idx = ct + it * kKThreads;
          const int key = idx >> 4, c8 = idx & 15, d0 = c8 * 8, pan = c8 >> 3, cc = c8 & 7;
          const bool live = n0 + key < wk.hi;
          const int g = d0 / GS;
          const uint16_t* srow = reinterpret_cast<const uint16_t*>(st + Raw::O_KS) + key * G::NG;
          const uint16_t* brow = reinterpret_cast<const uint16_t*>(st + Raw::O_KB) + key * G::NG;
          const float sc = dt_to_f<false>(srow[g]), bi = dt_to_f<false>(brow[g]);
          float c[8];
          load_codes8<BITS>(st + Raw::O_KP + key * G::KRB, d0, c);
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float2 w = __ffma2_rn(make_float2(sc, sc), make_float2(c[2 * i], c[2 * i + 1]),
                                        make_float2(bi, bi));
            const __half2 h = __floats2half2_rn(w.x, w.y);
            const float2 hf = __half22float2(h);
            const __half2 lo = __floats2half2_rn(w.x - hf.x, w.y - hf.y);
            hw[i] = live ? *reinterpret_cast<const uint32_t*>(&h) : 0u;
            lw[i] = live ? *reinterpret_cast<const uint32_t*>(&lo) : 0u;
          }
          const uint32_t off = pan * kPanelK + sw128(key, cc * 8);
          *reinterpret_cast<uint4*>(khi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(klo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bar.k_ready[buf]);
          mbar_arrive(&bar.raw_empty[s]);
        }
      }
      wk.advance();
    }
  } else if (v_warp_index(warp) >= 0) {
    // ---------------- V dequantisation: fp16(s*c + b), one HFMA2 per pair ----------------
    const int ct = v_warp_index(warp) * 32 + lane;
    constexpr int kVThreads = kVWarps * 32;
    int tc = 0;
    while (!hung && wk.next(p)) {
      for (int j = wk.sj; j < wk.j1 && !hung; j++, tc++) {
        const int s = tc % kRaw2, buf = tc & 1;
        const int n0 = wk.lo + j * kKT;
        const uint8_t* st = sm + LY::RAW + s * Raw::STAGE;
        if (!wait_all(&bar.raw_full[s], (uint32_t)((tc / kRaw2) & 1))) break;
        if (tc >= 2 && !wait_all(&bar.v_free[buf], (uint32_t)(((tc >> 1) & 1) ^ 1))) break;
        uint8_t* vt = sm + LY::V + buf * LY::VBUF;
#pragma unroll 4
        for (int it = 0; it < (kKT * 16) / kVThreads; it++) {
          const int idx = ct + it * kVThreads;
          const int key = idx >> 4, c8 = idx & 15, d0 = c8 * 8, pan = c8 >> 3, cc = c8 & 7;
          const bool live = n0 + key < wk.hi;
          const int g = d0 / GS;
          const uint16_t* srow = reinterpret_cast<const uint16_t*>(st + Raw::O_VS) + key * G::NG;
          const uint16_t* brow = reinterpret_cast<const uint16_t*>(st + Raw::O_VB) + key * G::NG;
          const __half2 s2 = __half2half2(__ushort_as_half(srow[g]));
          const __half2 b2 = __half2half2(__ushort_as_half(brow[g]));
          uint32_t cw[4];  // code pairs (2i, 2i + 1) as fp16 1024 + c
          if constexpr (BITS == 8) {
            const uint2 w = *reinterpret_cast<const uint2*>(st + Raw::O_VP + key * G::KRB + d0);
            cw[0] = prmt(w.x, 0x64006400u, 0x7150u);
            cw[1] = prmt(w.x, 0x64006400u, 0x7352u);
            cw[2] = prmt(w.y, 0x64006400u, 0x7150u);
            cw[3] = prmt(w.y, 0x64006400u, 0x7352u);
          } else {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(st + Raw::O_VP + key * G::KRB + d0 / 2);
#pragma unroll
            for (int i = 0; i < 4; i++)
              cw[i] = ((w >> (8 * i)) & 0xFu) | (((w >> (8 * i + 4)) & 0xFu) << 16) | 0x64006400u;
          }
          uint32_t vw[4];
          const __half2 k1024 = __float2half2_rn(1024.0f);
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const __half2 c2 = __hsub2(*reinterpret_cast<const __half2*>(&cw[i]), k1024);
            const __half2 h = __hfma2(s2, c2, b2);
            vw[i] = live ? *reinterpret_cast<const uint32_t*>(&h) : 0u;
          }
          *reinterpret_cast<uint4*>(vt + pan * kPanelK + sw128(key, cc * 8)) =
              make_uint4(vw[0], vw[1], vw[2], vw[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bar.v_ready[buf]);
          mbar_arrive(&bar.raw_empty[s]);
        }
      }
      wk.advance();
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue: lane 0 alone ----------------
    // Two walkers over the CTA's tiles: QK^T runs up to two tiles ahead of
    // PV (three S buffers), so the softmax of tile t + 1 never waits for the
    // PV of tile t - 1 to be issued.  At a unit boundary QK^T holds until
    // every PV of the unit is issued: the next unit's Q is written by the
    // softmax warps after they finish the unit.
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_f16(kRows, kKT, 0);
      const uint32_t idesc_pv = idesc_f16(kRows, 64, 1);
      // descriptors of the tile bases; a k-step or panel adds its byte
      // offset / 16 to the start-address field (all of shared memory fits it)
      const uint64_t dq = desc_sw128(smem_u32(sm + LY::Q));
      const uint64_t dk0 = desc_sw128(smem_u32(sm + LY::K));
      const uint64_t dv0 = desc_sw128(smem_u32(sm + LY::V));
      struct Cursor {
        Walk w;
        int j, t, u, t_first;
        bool valid;
      };
      auto start_cursor = [&](Cursor& c) {
        c.w = wk;
        c.valid = c.w.next(p);
        c.j = c.w.sj;
        c.t = c.t_first = c.u = 0;
      };
      auto step_cursor = [&](Cursor& c) {
        c.j++;
        c.t++;
        if (c.j == c.w.j1) {
          c.w.advance();
          c.u++;
          c.valid = c.w.next(p);
          if (c.valid) {
            c.j = c.w.sj;
            c.t_first = c.t;
          }
        }
      };
      Cursor cq, cp;
      start_cursor(cq);
      start_cursor(cp);
      bool ok = true;
      while (ok && (cq.valid || cp.t < cq.t)) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        if (cq.valid && cq.t <= cp.t + 2 && cq.u == cp.u) {
          const int t = cq.t;
          if ((t == cq.t_first && !mbar_wait(bar.q_ready, (uint32_t)(cq.u & 1))) ||
              !mbar_wait(&bar.k_ready[t & 1], (uint32_t)((t >> 1) & 1)) ||
              (t >= kSBuf && !mbar_wait(&bar.pv_done[t % kSBuf], (uint32_t)(((t / kSBuf) & 1) ^ 1)))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t dk = dk0 + (uint64_t)(((t & 1) * LY::KBUF) >> 4);
          const uint32_t dS = tm + (uint32_t)((t % kSBuf) * 64);
#pragma unroll
          for (int part = 0; part < 2; part++)  // hi, then lo
#pragma unroll
            for (int ks = 0; ks < TD / 16; ks++) {
              const int pan = ks >> 2, kk = ks & 3;
              umma_ss(dS, dq + (uint64_t)((pan * kPanelQ + 32 * kk) >> 4),
                      dk + (uint64_t)((part * 2 * kPanelK + pan * kPanelK + 32 * kk) >> 4),
                      idesc_qk, (part | ks) ? 1u : 0u);
            }
          umma_commit(&bar.s_full[t % kSBuf]);
          umma_commit(&bar.k_free[t & 1]);
          step_cursor(cq);
          continue;
        }
        // PV of the oldest tile whose QK^T is issued
        const int t = cp.t;
        const bool first = t == cp.t_first;
        if (!mbar_wait(&bar.p_ready[t % kSBuf], (uint32_t)((t / kSBuf) & 1)) ||
            !mbar_wait(&bar.v_ready[t & 1], (uint32_t)((t >> 1) & 1)) ||
            (first && cp.u > 0 && !mbar_wait(bar.o_free, (uint32_t)((cp.u - 1) & 1)))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t dv = dv0 + (uint64_t)(((t & 1) * LY::VBUF) >> 4);
#pragma unroll
        for (int ks = 0; ks < kKT / 16; ks++)
#pragma unroll
          for (int pd = 0; pd < 2; pd++)
            umma_ts(tm + kTmO + pd * 64, tm + (uint32_t)((t % kSBuf) * 64 + 8 * ks),
                    dv + (uint64_t)((pd * kPanelK + 2048 * ks) >> 4), idesc_pv,
                    (first && ks == 0) ? 0u : 1u);
        umma_commit(&bar.pv_done[t % kSBuf]);
        umma_commit(&bar.v_free[t & 1]);
        step_cursor(cp);
      }
      if (!ok) {
        hung = true;
        *abort_flag = 1;
      }
      // every issued MMA has finished before the TMEM is released
      umma_commit(bar.mma_end);
      mbar_wait(bar.mma_end, 0u);
    }
    __syncwarp();
  } else {
    // ---------------- softmax (warps 0-7) ----------------
    const int kh = warp >> 2;              // key half of every tile (and d panel of O)
    const int r = (warp & 3) * 32 + lane;  // query row, TMEM lane
    const uint32_t lane_base = tm + ((uint32_t)((warp & 3) * 32) << 16);
    const int pair_bar = 2 + (warp & 3);   // named barrier of warps w and w + 4
    int tc = 0, units = 0;
    bool bad = false;
    while (!hung && wk.next(p)) {
      const int b = (int)(wk.hp / p.Hkv), kvh = (int)(wk.hp - (int64_t)b * p.Hkv);
      const int qr = wk.qt * kRows + r;
      const bool qvalid = qr < qrows;
      const int l = qvalid ? qr / nrep : 0, hh = qvalid ? qr - l * nrep : 0;
      const int pos = wk.Nb - L + l;
      int klo = 0, khi = wk.Nb - 1;
      if (p.mask_mode == 1) {
        khi = min(khi, pos);
        if (p.window > 0) klo = max(0, pos - p.window + 1);
      }
      const bool partial = wk.sj > 0 || wk.j1 < wk.ntl;
      // ---- Q: q * dtype(scale) rounded, this half's d panel (the previous
      // unit's QK^T finished: its last S was read) ----
      {
        const float scale_dt = round_dt<false>(p.scale);
        const uint16_t* qrow = p.q + (((int64_t)b * p.Hq + kvh * nrep + hh) * L + l) * TD + kh * 64;
        uint8_t* qp = sm + LY::Q + kh * kPanelQ;
#pragma unroll
        for (int c8 = 0; c8 < 8; c8++) {
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          if (qvalid) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qrow + c8 * 8));
            const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const float a0 = round_dt<false>(dt_to_f<false>((uint16_t)(rw[k] & 0xffffu)) * scale_dt);
              const float a1 = round_dt<false>(dt_to_f<false>((uint16_t)(rw[k] >> 16)) * scale_dt);
              w[k] = pack_h2(a0, a1);
            }
          }
          *reinterpret_cast<uint4*>(qp + sw128(r, c8 * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.q_ready);
      }
      float m_used = kNeg, lsum = 0.0f;
      const int t0 = tc;
      // `bad`: a bounded wait of this warp gave up since the last pair
      // barrier; the pair barrier turns it into a joint exit.
      for (int j = wk.sj; j < wk.j1; j++, tc++) {
        const int sb = tc % kSBuf;
        const int n0 = wk.lo + j * kKT + kh * 32;  // this thread's first key
        bool ok = !bad && !*abort_flag && mbar_wait(&bar.s_full[sb], (uint32_t)((tc / kSBuf) & 1));
        ok = __all_sync(0xffffffffu, ok);
        uint32_t x[32];
        float tmax = kNeg;
        const bool fast =
            __all_sync(0xffffffffu, qvalid && n0 >= klo && n0 + 31 <= khi && n0 + 32 <= wk.hi);
        if (ok) {
          tc_fence_after();
          tmem_ld32(lane_base + (uint32_t)(sb * 64 + kh * 32), x);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            float a, c;
            round_dt2<false>(__uint_as_float(x[k]), __uint_as_float(x[k + 1]), a, c);
            if (!fast) {
              const int n = n0 + k;
              a = (qvalid && n < wk.hi && n >= klo && n <= khi) ? a : kNeg;
              c = (qvalid && n + 1 < wk.hi && n + 1 >= klo && n + 1 <= khi) ? c : kNeg;
            }
            tmax = fmaxf(tmax, fmaxf(a, c));
            x[k] = __float_as_uint(a);
            x[k + 1] = __float_as_uint(c);
          }
        }
        float* xc = xch + (tc & 1) * 2 * kRows;
        xc[kh * kRows + r] = tmax;
        if (!pair_and(pair_bar, ok)) {
          hung = true;
          break;
        }
        tmax = fmaxf(xc[r], xc[kRows + r]);
        // lazy rescale: only when a row's maximum grows by more than 2^8
        const bool want = tmax > m_used && ((tmax - m_used) * kLog2e > 8.0f || m_used == kNeg);
        if (__any_sync(0xffffffffu, want)) {
          const float alpha = want ? ex2((m_used - tmax) * kLog2e) : 1.0f;
          lsum *= alpha;
          if (tc > t0) {  // O holds this unit's earlier tiles: wait for PV(t - 1)
            const bool okp = __all_sync(
                0xffffffffu, mbar_wait(&bar.pv_done[(tc - 1) % kSBuf], (uint32_t)(((tc - 1) / kSBuf) & 1)));
            if (!okp) {
              bad = true;
            } else {
              tc_fence_after();
#pragma unroll 1
              for (int c0 = 0; c0 < 64; c0 += 32) {
                uint32_t o[32];
                tmem_ld32(lane_base + kTmO + kh * 64 + c0, o);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                tmem_st32(lane_base + kTmO + kh * 64 + c0, o);
              }
              tmem_wait_st();
            }
          }
          if (want) m_used = tmax;
        }
        if (bad) continue;  // the next pair barrier ends the loop for both warps
        const float mls = m_used * kLog2e;
        uint32_t pw[16];
        float2 ls2 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const float2 arg = __ffma2_rn(make_float2(__uint_as_float(x[k]), __uint_as_float(x[k + 1])),
                                        make_float2(kLog2e, kLog2e), make_float2(-mls, -mls));
          float2 pv = make_float2(ex2(arg.x), ex2(arg.y));
          if (!fast) {  // masked keys carry the kNeg sentinel: p = 0
            pv.x = x[k] != __float_as_uint(kNeg) ? pv.x : 0.0f;
            pv.y = x[k + 1] != __float_as_uint(kNeg) ? pv.y : 0.0f;
          }
          ls2 = __fadd2_rn(ls2, pv);
          pw[k / 2] = pack_h2(pv.x, pv.y);
        }
        lsum += ls2.x + ls2.y;
        tmem_st16(lane_base + (uint32_t)(sb * 64 + kh * 16), pw);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar.p_ready[sb]);
      }
      if (hung) break;
      // ---- epilogue: out = O / l (half kh writes d panel kh) ----
      xl[kh * kRows + r] = lsum;
      if (!pair_and(pair_bar, !bad)) {
        hung = true;
        break;
      }
      const float lt = xl[r] + xl[kRows + r];
      const int tl = tc - 1;  // the unit's last tile
      bad = !__all_sync(0xffffffffu, mbar_wait(&bar.pv_done[tl % kSBuf], (uint32_t)((tl / kSBuf) & 1)));
      if (!bad) {
        tc_fence_after();
        if (!partial) {
          const int64_t orow = ((int64_t)b * p.Hq + kvh * nrep + hh) * L + l;
          uint16_t* dst = p.out + orow * TD + kh * 64;
#pragma unroll 1
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(lane_base + kTmO + kh * 64 + c0, o);
            tmem_wait_ld();
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
            uint32_t w[16];
#pragma unroll
            for (int k = 0; k < 32; k += 2)
              w[k / 2] = pack_h2(__uint_as_float(o[k]) * inv, __uint_as_float(o[k + 1]) * inv);
            if (qvalid) {
#pragma unroll
              for (int k = 0; k < 16; k += 4)
                *reinterpret_cast<uint4*>(dst + c0 + 2 * k) = make_uint4(w[k], w[k + 1], w[k + 2], w[k + 3]);
            }
          }
        } else {
          // partial row of a unit cut between CTAs: [m, l, 0, 0, O(128)] in
          // slot 2c (the CTA's first unit) or 2c + 1 (its last)
          float* srow = p.ws_o + (((size_t)blockIdx.x * 2 + (units ? 1 : 0)) * kRows + r) * kSlotRow;
#pragma unroll 1
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(lane_base + kTmO + kh * 64 + c0, o);
            tmem_wait_ld();
            if (qvalid) {
#pragma unroll
              for (int k = 0; k < 32; k += 4)
                *reinterpret_cast<float4*>(srow + 4 + kh * 64 + c0 + k) =
                    make_float4(__uint_as_float(o[k]), __uint_as_float(o[k + 1]),
                                __uint_as_float(o[k + 2]), __uint_as_float(o[k + 3]));
            }
          }
          if (qvalid) {
            if (kh == 0) {
              srow[0] = m_used;
              srow[1] = lt;
            }
            srow[2 + kh] = 0.0f;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.o_free);
      units++;
      wk.advance();
    }
  }
  if (hung && lane == 0) atomicExch(p.err, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(512));
  }
}

template <int BITS, int GS>
int32_t launch_tc2(Params& p, int B, void* ws, size_t ws_bytes, cudaStream_t st) {
  auto kern = prefill_tc2_kernel<BITS, GS>;
  constexpr int smem = Lay2<BITS, GS>::TOTAL;
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  int32_t rc = kernel_setup(reinterpret_cast<const void*>(kern), kThreads2, smem, dev, nullptr);
  if (rc) return rc;
  const int qrows = p.nrep * p.L;
  const int nqb = (qrows + kRows - 1) / kRows;
  int64_t ctas = 0, Th = 0;
  size_t need = kPartialOff;
  if (!p.seq_lens) {
    for (int q = 0; q < nqb; q++)
      Th += tc_block_tiles<kKT>(q, p.N, p.L, p.nrep, p.mask_mode, p.window);
    const int64_t T = (int64_t)B * p.Hkv * Th;
    ctas = std::min<int64_t>(num_sms(dev), T);
    need = kPartialOff + (size_t)2 * ctas * kRows * kSlotRow * sizeof(float);
    if (Th > INT32_MAX || (ws && ws_bytes < need)) {
      ctas = 0;
      need = kPartialOff;
    }
  }
  if (!ws) {
    ws = managed_workspace(dev, need, st, &rc);
    if (rc) return rc;
  }
  p.err = static_cast<int*>(ws);
  p.QB = (int)ctas;
  p.Tu = (int)Th;
  p.ws_o = ctas > 0 ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kPartialOff) : nullptr;
  if (ctas > 0) {
    KVQ_CUDA_TRY(launch_pdl(kern, dim3((unsigned)ctas), dim3(kThreads2), (size_t)smem, st, p));
    KVQ_CUDA_TRY(launch_pdl(prefill_tc_merge_kernel<false, kKT>, dim3((unsigned)ctas),
                            dim3(kMergeThreads), 0, st, p));
    return KVQ_OK;
  }
  const dim3 grid((unsigned)nqb, (unsigned)p.Hkv, (unsigned)B);
  KVQ_CUDA_TRY(launch_pdl(kern, grid, dim3(kThreads2), (size_t)smem, st, p));
  return KVQ_OK;
}

}  // namespace

bool prefill_tc2_supported(int bits, int D, int gs, int dtype, int L) {
  return (bits == 4 || bits == 8) && D == TD && (gs == 32 || gs == 64 || gs == 128) &&
         dtype == KVQ_DTYPE_FLOAT16 && L > 1;
}

int32_t launch_prefill_tc2(Params& p, int B, int bits, int gs, void* ws, size_t ws_bytes,
                           cudaStream_t st) {
  if (bits == 8) {
    if (gs == 32) return launch_tc2<8, 32>(p, B, ws, ws_bytes, st);
    if (gs == 64) return launch_tc2<8, 64>(p, B, ws, ws_bytes, st);
    return launch_tc2<8, 128>(p, B, ws, ws_bytes, st);
  }
  if (gs == 32) return launch_tc2<4, 32>(p, B, ws, ws_bytes, st);
  if (gs == 64) return launch_tc2<4, 64>(p, B, ws, ws_bytes, st);
  return launch_tc2<4, 128>(p, B, ws, ws_bytes, st);
}

}  // namespace attn
}  // namespace kvq
