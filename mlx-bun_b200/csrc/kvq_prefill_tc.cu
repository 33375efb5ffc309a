// kvq_prefill_tc.cu — chunked prefill attention on the 5th-generation tensor
// cores (tcgen05 / UMMA with TMEM accumulators) for 8-bit codes, D = 128,
// group 64 (the config-4 shape); other shapes take the split kernel.
//
// A unit is 128 query rows of one (batch, kv head): rows are (position,
// head) pairs of the GQA group (row qr -> position qr / nrep, head qr %
// nrep), so every key tile serves all query heads that share it.  Query
// row r is the row of TMEM lane r, so the online softmax needs no cross-lane
// traffic.  A ninth warp streams the key rows in tiles of 128 with 1-D TMA
// bulk copies (the decode ring).  Two of the 8 softmax warps share each row
// (warps w and w + 4 reach the same TMEM lanes), each taking half of every
// key tile; they exchange the tile maximum and, at the end, their sums
// through shared memory.
//
// Per key tile:
//   1. the codes become fp16 subnormals (code * 2^-24, exact) in shared
//      memory, 128-byte-swizzled rows of 64 d: the K tile is the K-major B
//      operand of QK^T, the V tile (same layout, two buffers) the MN-major B
//      operand of PV;
//   2. QK^T per quantisation group g: S_g = Q_g . C_g^T (M 128, N 128, K 64)
//      into TMEM (qdot factoring: logit = sum_g ks*2^24*S_g + kb*sum(q_g)),
//      issued once the K tile is converted and running while V is;
//   3. softmax, two passes over TMEM: logits rounded to the dtype and masked
//      (written back over S_0) with the tile maximum, then p = 2^((x - m)
//      log2 e) against the row's running maximum m, P'_g = fp16(p * vs_g)
//      into TMEM (the A operand of PV) and sum(p * vb_g) in registers.  O is
//      rescaled only when the maximum grows by more than 2^8 (lazy rescale:
//      P' stays far inside fp16, the final O / l is the same);
//   4. PV per group: O_g += P'_g . V_g (M 128, N 64, K 128) in TMEM.
// QK of tile j + 1 waits on its commit, which also covers PV(j); with V in
// two buffers, PV(j) runs on while tile j + 1's codes are converted.  Every
// wait is bounded; on timeout the kernel raises the device error flag and
// skips the rest of its tiles.
//
// Grid: without per-sequence key counts, one CTA per SM, each taking an
// equal run of the key tiles of all units (b, kv head, query block) laid end
// to end; a unit cut between CTAs leaves partial (m, l, sum(p vb_g), O) rows
// that prefill_tc_merge_kernel combines.  Otherwise one CTA per unit.
//
// TMEM (512 columns, one CTA per SM): S_0 [0,128) S_1 [128,256) P'_0
// [256,320) P'_1 [320,384) O_0 [384,448) O_1 [448,512).
#include "kvq_tc.cuh"

namespace kvq {
namespace attn {
namespace {

using namespace tc;

constexpr int kKeys = 128;     // keys per tile
constexpr int kTcStages = 2;   // raw TMA ring stages
constexpr int TGS = 64, TNG = 2;

// shared memory (offsets from a 1024-byte aligned base)
constexpr int kQOff = 0;                        // [TNG] SW128 [128 rows][64] fp16
constexpr int kKcOff = kQOff + TNG * 16384;     // [TNG] SW128 [128 keys][64] fp16
constexpr int kVcOff = kKcOff + TNG * 16384;    // [2 tiles][TNG] SW128 [128 keys][64] fp16
constexpr int kVcTile = TNG * 16384;            // V of tile j sits in buffer j & 1
constexpr int kSclOff = kVcOff + 2 * kVcTile;   // f32 [4][TNG][128]: ks*2^24, kb, vs, vb
constexpr int kRawOff = kSclOff + 4 * TNG * kKeys * 4;
using RawLay = StageLayout<8, TD, TGS, kKeys>;
constexpr int kXchOff = kRawOff + kTcStages * RawLay::STAGE;  // f32 [2][4][128] row exchange
constexpr int kBarOff = kXchOff + 2 * 4 * kRows * 4;          // full[2], empty[2], qk, pv
constexpr int kCtlOff = kBarOff + (2 * kTcStages + 2) * 8;   // tmem base, abort flag
constexpr int kTcSmem = kCtlOff + 16 + 1024;                  // + alignment slack
static_assert(kTcSmem <= 227 * 1024, "prefill tile buffers exceed the shared memory of a CTA");
constexpr int kCWarps = 8;                                    // softmax warps: 2 per query row
constexpr int kCThreads = kCWarps * 32;

// 8 byte codes (two words) as four fp16-subnormal pairs (code in the low
// mantissa bits, exponent zero)
__device__ __forceinline__ uint4 codes8_to_f16(uint32_t w0, uint32_t w1) {
  uint4 r;
  r.x = prmt(w0, 0u, 0x4140u);
  r.y = prmt(w0, 0u, 0x4342u);
  r.z = prmt(w1, 0u, 0x4140u);
  r.w = prmt(w1, 0u, 0x4342u);
  return r;
}

template <bool BF>
__global__ void __launch_bounds__(288, 1) prefill_tc_kernel(const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kBarOff);
  uint64_t* empty = full + kTcStages;
  uint64_t* qk_bar = empty + kTcStages;
  uint64_t* pv_bar = qk_bar + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sm + kCtlOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kCtlOff + 4);
  float* scl = reinterpret_cast<float*>(sm + kSclOff);  // [4][TNG][128]
  float* xch = reinterpret_cast<float*>(sm + kXchOff);  // [2 halves][4][128] row exchange

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool producer = warp == kCWarps;
  const int nrep = p.nrep, L = p.L, qrows = nrep * L;
  const int nqb = (qrows + kRows - 1) / kRows;
  // Work of this CTA: the key tiles [T0, T1) of the units (b, kv head, query
  // block) laid end to end (b, then kv head, then query block), starting in
  // pair hp0 = b * Hkv + kv head at query block qt0, tile j00 of that block.
  // Balanced grid (p.QB CTAs): equal runs of the whole list.  Otherwise one
  // CTA per unit, (blockIdx.x, .y, .z) = (query block, kv head, b).
  int Nb = p.N;
  int64_t T0, T1, hp0;
  int qt0, j00;
  if (p.QB > 0) {
    const int64_t T = (int64_t)p.B * p.Hkv * p.Tu;
    T0 = (int64_t)blockIdx.x * T / p.QB;
    T1 = (int64_t)(blockIdx.x + 1) * T / p.QB;
    hp0 = T0 / p.Tu;
    tc_locate<kKeys>((int)(T0 - hp0 * p.Tu), nqb, Nb, L, nrep, p.mask_mode, p.window, lane, qt0, j00);
  } else {
    hp0 = (int64_t)blockIdx.z * p.Hkv + blockIdx.y;
    qt0 = blockIdx.x;
    j00 = 0;
    if (p.seq_lens) Nb = min(max(p.seq_lens[blockIdx.z], 0), p.N);
    T0 = 0;
    T1 = tc_block_tiles<kKeys>(qt0, Nb, L, nrep, p.mask_mode, p.window);
  }

  if (tid == 0) {
    for (int s = 0; s < kTcStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    mbar_init(qk_bar, 1);
    mbar_init(pv_bar, 1);
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

  if (producer) {
    if (lane == 0) {
      int tcount = 0;
      int64_t t = T0, hp = hp0;
      int qt = qt0, sj = j00;
      bool first = true;
      while (!hung && (first || t < T1)) {
        first = false;
        int lo, hi;
        const int ntl = tc_block_tiles<kKeys>(qt, Nb, L, nrep, p.mask_mode, p.window, &lo, &hi);
        const int j1 = (int)min((int64_t)ntl, (int64_t)sj + (T1 - t));
        const int b = (int)(hp / p.Hkv), kvh = (int)(hp - (int64_t)b * p.Hkv);
        const int64_t kbase = (int64_t)b * p.k_bstride + (int64_t)kvh * p.k_hstride;
        const int64_t vbase = (int64_t)b * p.v_bstride + (int64_t)kvh * p.v_hstride;
        for (int j = sj; j < j1; j++, tcount++) {
          const int s = tcount % kTcStages;
          if (tcount >= kTcStages &&
              (*abort_flag || !mbar_wait(&empty[s], (uint32_t)(((tcount / kTcStages) & 1) ^ 1)))) {
            hung = true;
            *abort_flag = 1;
            break;
          }
          const int row = lo + j * kKeys;
          const int rows = min(kKeys, hi - row);
          issue_chunk<8, TD, TGS, kKeys>(p, sm + kRawOff + s * RawLay::STAGE, &full[s], kbase, vbase,
                                         row, (uint32_t)((rows + kTile - 1) / kTile * kTile));
        }
        t += j1 - sj;
        sj = 0;
        if (++qt == nqb) {
          qt = 0;
          ++hp;
        }
      }
    }
  } else {
    // Two threads per query row: warps w and w + 4 share TMEM lanes 32(w%4)..
    // and take the first / second half of every key tile (and, at the end,
    // of the output columns: half kh owns group kh's d).
    const int kh = warp >> 2;                  // key half
    const int r = (warp & 3) * 32 + lane;      // query row, TMEM lane
    const uint32_t lane_base = tm + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t idesc_qk = idesc_f16(kRows, kKeys, 0);
    const uint32_t idesc_pv = idesc_f16(kRows, TGS, 1);
    const int kbeg = kh * (kKeys / 2);  // this thread's keys in a tile: [kbeg, kbeg + 64)
    int tcount = 0, seg = 0;  // tiles streamed so far (ring stage, barrier phases), units done
    int64_t t = T0, hp = hp0;
    int qt = qt0, sj = j00;
    bool first = true;
    while (first || t < T1) {
      first = false;
      int lo, hi;
      const int ntl = tc_block_tiles<kKeys>(qt, Nb, L, nrep, p.mask_mode, p.window, &lo, &hi);
      const int j1 = (int)min((int64_t)ntl, (int64_t)sj + (T1 - t));  // this CTA's tiles [sj, j1)
      const int b = (int)(hp / p.Hkv), kvh = (int)(hp - (int64_t)b * p.Hkv);
      const bool partial = sj > 0 || j1 < ntl;
      const int qr0 = qt * kRows;
      const int qr = qr0 + r;
      const bool qvalid = qr < qrows;
      const int l = qvalid ? qr / nrep : 0, hh = qvalid ? qr - l * nrep : 0;
      const int pos = Nb - L + l;  // key position of this query row (bottom-right aligned)
      int klo = 0, khi = Nb - 1;
      if (p.mask_mode == 1) {
        khi = min(khi, pos);
        if (p.window > 0) klo = max(0, pos - p.window + 1);
      }
      // ---- query row (half kh writes group kh): q * dtype(scale) rounded to the dtype ----
      float qs[TNG];
      {
        const float scale_dt = round_dt<BF>(p.scale);
        const uint16_t* qrow = p.q + (((int64_t)b * p.Hq + kvh * nrep + hh) * L + l) * TD;
#pragma unroll
        for (int g = 0; g < TNG; g++) {
          uint8_t* qg = sm + kQOff + g * 16384;
          float sum = 0.0f;
#pragma unroll
          for (int c8 = 0; c8 < 8; c8++) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const int d = g * TGS + c8 * 8 + 2 * j;
              const float a0 = qvalid ? round_dt<BF>(dt_to_f<BF>(__ldg(qrow + d)) * scale_dt) : 0.0f;
              const float a1 = qvalid ? round_dt<BF>(dt_to_f<BF>(__ldg(qrow + d + 1)) * scale_dt) : 0.0f;
              sum += a0 + a1;
              w[j] = pack_h2(a0, a1);
            }
            if (g == kh)
              *reinterpret_cast<uint4*>(qg + sw128(r, c8 * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
          qs[g] = sum;
        }
      }
      float m_used = kNeg, lsum = 0.0f, pbs[TNG] = {0.0f, 0.0f};

      for (int j = sj; j < j1; j++, tcount++) {
        const int s = tcount % kTcStages;
        const int n0 = lo + j * kKeys;
        // ---- 1. codes -> fp16 subnormals (K and V), scales -> f32 ----
        {
          const bool ok = !hung && !*abort_flag && mbar_wait(&full[s], (uint32_t)((tcount / kTcStages) & 1));
          if (!__all_sync(0xffffffffu, ok)) {
            if (!hung && lane == 0) *abort_flag = 1;
            hung = true;
          }
        }
        // K codes and all scales first; QK^T is issued as soon as the K tile is
        // in place and runs while V is converted.  V of the tile with stream
        // index t goes to buffer t & 1: PV(t - 1) may still read the other one,
        // and PV(t - 2), the last reader of this one, completed under the QK
        // commit of tile t - 1.
        const uint8_t* st = sm + kRawOff + s * RawLay::STAGE;
        uint8_t* vc = sm + kVcOff + (tcount & 1) * kVcTile;
        if (!hung) {
#pragma unroll 4
          for (int it = 0; it < (kKeys * TNG * 8) / kCThreads; it++) {
            const int idx = tid + it * kCThreads;
            const int key = idx >> 4, g = (idx >> 3) & 1, c8 = idx & 7;
            const uint2 kw = *reinterpret_cast<const uint2*>(st + RawLay::O_KP + key * TD + g * TGS + c8 * 8);
            *reinterpret_cast<uint4*>(sm + kKcOff + g * 16384 + sw128(key, c8 * 8)) = codes8_to_f16(kw.x, kw.y);
          }
          {
            // thread t: key t & 127, arrays (K scale+bias) or (V scale+bias) by t >> 7;
            // keys past the range hold stale ring bytes and get 0
            const int key = tid & (kKeys - 1), which = tid >> 7;
            const bool live = n0 + key < hi;
            const int oa = which ? RawLay::O_VS : RawLay::O_KS, ob = which ? RawLay::O_VB : RawLay::O_KB;
            const uint32_t sw = live ? *reinterpret_cast<const uint32_t*>(st + oa + key * 4) : 0u;
            const uint32_t bw = live ? *reinterpret_cast<const uint32_t*>(st + ob + key * 4) : 0u;
#pragma unroll
            for (int g = 0; g < TNG; g++) {
              const float sv = dt_to_f<BF>((uint16_t)(g ? (sw >> 16) : (sw & 0xffffu)));
              const float bv = dt_to_f<BF>((uint16_t)(g ? (bw >> 16) : (bw & 0xffffu)));
              scl[((which * 2 + 0) * TNG + g) * kKeys + key] = which ? sv : sv * kCodeUnitInv;
              scl[((which * 2 + 1) * TNG + g) * kKeys + key] = bv;
            }
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        asm volatile("bar.sync 1, %0;" ::"r"(kCThreads) : "memory");
        tc_fence_after();

        // ---- 2. S_g = Q_g . C_g^T ----
        if (tid == 0 && !hung && !*abort_flag) {
#pragma unroll
          for (int g = 0; g < TNG; g++)
#pragma unroll
            for (int ks = 0; ks < TGS / 16; ks++)
              umma_ss(tm + g * 128, desc_sw128(smem_u32(sm + kQOff + g * 16384) + 32 * ks),
                      desc_sw128(smem_u32(sm + kKcOff + g * 16384) + 32 * ks), idesc_qk,
                      ks > 0 ? 1u : 0u);
          umma_commit(qk_bar);
        }
        if (!hung) {
#pragma unroll 4
          for (int it = 0; it < (kKeys * TNG * 8) / kCThreads; it++) {
            const int idx = tid + it * kCThreads;
            const int key = idx >> 4, g = (idx >> 3) & 1, c8 = idx & 7;
            const uint2 vw = *reinterpret_cast<const uint2*>(st + RawLay::O_VP + key * TD + g * TGS + c8 * 8);
            *reinterpret_cast<uint4*>(vc + g * 16384 + sw128(key, c8 * 8)) = codes8_to_f16(vw.x, vw.y);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // raw stage free
        // the V tile is read by PV after the barrier that ends step 3c
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        {
          // this commit also covers the previous PV: after it, P' and O are free
          const bool ok = !hung && !*abort_flag && mbar_wait(qk_bar, (uint32_t)(tcount & 1));
          if (!__all_sync(0xffffffffu, ok)) {
            if (!hung && lane == 0) *abort_flag = 1;
            hung = true;
          }
        }
        tc_fence_after();

        // every key of this thread's half valid for this row (warp-uniform test)?
        const bool fast = __all_sync(0xffffffffu, qvalid && n0 + kbeg >= klo &&
                                                      n0 + kbeg + kKeys / 2 - 1 <= khi &&
                                                      n0 + kbeg + kKeys / 2 <= hi);
        // ---- 3a. logits (rounded, masked) over S_0, half-tile maximum ----
        float tmax = kNeg;
        if (!hung) {
#pragma unroll 1
          for (int c0 = kbeg; c0 < kbeg + kKeys / 2; c0 += 32) {
            uint32_t s0[32], s1[32];
            tmem_ld32(lane_base + 0 + c0, s0);
            tmem_ld32(lane_base + 128 + c0, s1);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; k += 4) {
              // two keys per paired-lane fma (each lane the same IEEE fma as a scalar one)
              const float4 ks0 = *reinterpret_cast<const float4*>(scl + (0 * TNG + 0) * kKeys + c0 + k);
              const float4 ks1 = *reinterpret_cast<const float4*>(scl + (0 * TNG + 1) * kKeys + c0 + k);
              const float4 kb0 = *reinterpret_cast<const float4*>(scl + (1 * TNG + 0) * kKeys + c0 + k);
              const float4 kb1 = *reinterpret_cast<const float4*>(scl + (1 * TNG + 1) * kKeys + c0 + k);
              const float2 q0 = make_float2(qs[0], qs[0]), q1 = make_float2(qs[1], qs[1]);
              float sc[4];
#pragma unroll
              for (int h2 = 0; h2 < 2; h2++) {
                const float2 a0 = h2 ? make_float2(ks0.z, ks0.w) : make_float2(ks0.x, ks0.y);
                const float2 a1 = h2 ? make_float2(ks1.z, ks1.w) : make_float2(ks1.x, ks1.y);
                const float2 b0 = h2 ? make_float2(kb0.z, kb0.w) : make_float2(kb0.x, kb0.y);
                const float2 b1 = h2 ? make_float2(kb1.z, kb1.w) : make_float2(kb1.x, kb1.y);
                const int u = k + 2 * h2;
                float2 t = __ffma2_rn(b0, q0, make_float2(0.0f, 0.0f));
                t = __ffma2_rn(a0, make_float2(__uint_as_float(s0[u]), __uint_as_float(s0[u + 1])), t);
                t = __ffma2_rn(b1, q1, t);
                t = __ffma2_rn(a1, make_float2(__uint_as_float(s1[u]), __uint_as_float(s1[u + 1])), t);
                sc[2 * h2] = t.x;
                sc[2 * h2 + 1] = t.y;
              }
              float x[4];
              round_dt2<BF>(sc[0], sc[1], x[0], x[1]);
              round_dt2<BF>(sc[2], sc[3], x[2], x[3]);
              if (!fast) {
#pragma unroll
                for (int u = 0; u < 4; u++) {
                  const int n = n0 + c0 + k + u;
                  x[u] = (qvalid && n < hi && n >= klo && n <= khi) ? x[u] : kNeg;
                }
              }
#pragma unroll
              for (int u = 0; u < 4; u++) {
                tmax = fmaxf(tmax, x[u]);
                s0[k + u] = __float_as_uint(x[u]);
              }
            }
            tmem_st32(lane_base + 0 + c0, s0);
          }
          tmem_wait_st();
        }
        // row maximum of the tile from both halves
        xch[(kh * 4 + 0) * kKeys + r] = tmax;
        asm volatile("bar.sync 1, %0;" ::"r"(kCThreads) : "memory");
        tmax = fmaxf(xch[(0 * 4 + 0) * kKeys + r], xch[(1 * 4 + 0) * kKeys + r]);

        // ---- 3b. lazy rescale: only when a row's maximum grows by more than
        // 2^8.  The decision is warp-uniform (tcgen05.ld / st are collective);
        // rows that need none scale by 1.  Half kh rescales group kh's O.
        const bool want = tmax > m_used && ((tmax - m_used) * kLog2e > 8.0f || m_used == kNeg);
        if (!hung && __any_sync(0xffffffffu, want)) {
          const float alpha = want ? ex2((m_used - tmax) * kLog2e) : 1.0f;
          lsum *= alpha;
#pragma unroll
          for (int g = 0; g < TNG; g++) pbs[g] *= alpha;
          if (j > sj) {
#pragma unroll 1
            for (int c0 = 0; c0 < TGS; c0 += 32) {
              uint32_t o[32];
              tmem_ld32(lane_base + 384 + kh * TGS + c0, o);
              tmem_wait_ld();
#pragma unroll
              for (int k = 0; k < 32; k++) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
              tmem_st32(lane_base + 384 + kh * TGS + c0, o);
            }
            tmem_wait_st();
          }
          if (want) m_used = tmax;
        }
        // ---- 3c. p, P'_g = fp16(p vs_g) into TMEM, l and sum(p vb_g) ----
        if (!hung) {
          const float mls = m_used * kLog2e;
#pragma unroll 1
          for (int c0 = kbeg; c0 < kbeg + kKeys / 2; c0 += 32) {
            uint32_t x[32];
            tmem_ld32(lane_base + 0 + c0, x);
            tmem_wait_ld();
            uint32_t pw0[16], pw1[16];
            float2 ls2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int k = 0; k < 32; k += 4) {
              const float4 vs0 = *reinterpret_cast<const float4*>(scl + (2 * TNG + 0) * kKeys + c0 + k);
              const float4 vs1 = *reinterpret_cast<const float4*>(scl + (2 * TNG + 1) * kKeys + c0 + k);
              const float4 vb0 = *reinterpret_cast<const float4*>(scl + (3 * TNG + 0) * kKeys + c0 + k);
              const float4 vb1 = *reinterpret_cast<const float4*>(scl + (3 * TNG + 1) * kKeys + c0 + k);
#pragma unroll
              for (int h2 = 0; h2 < 2; h2++) {
                const int kk = k + 2 * h2;
                const float2 arg = __ffma2_rn(
                    make_float2(__uint_as_float(x[kk]), __uint_as_float(x[kk + 1])),
                    make_float2(kLog2e, kLog2e), make_float2(-mls, -mls));
                float2 pv = make_float2(ex2(arg.x), ex2(arg.y));
                if (!fast) {
                  // masked keys carry the kNeg sentinel: p = 0 for them, even
                  // while the row's running maximum is still the sentinel
                  pv.x = x[kk] != __float_as_uint(kNeg) ? pv.x : 0.0f;
                  pv.y = x[kk + 1] != __float_as_uint(kNeg) ? pv.y : 0.0f;
                }
                ls2 = __fadd2_rn(ls2, pv);
                const float2 vsa = h2 ? make_float2(vs0.z, vs0.w) : make_float2(vs0.x, vs0.y);
                const float2 vsb = h2 ? make_float2(vs1.z, vs1.w) : make_float2(vs1.x, vs1.y);
                const float2 vba = h2 ? make_float2(vb0.z, vb0.w) : make_float2(vb0.x, vb0.y);
                const float2 vbb = h2 ? make_float2(vb1.z, vb1.w) : make_float2(vb1.x, vb1.y);
                pbs[0] = fmaf(pv.y, vba.y, fmaf(pv.x, vba.x, pbs[0]));
                pbs[1] = fmaf(pv.y, vbb.y, fmaf(pv.x, vbb.x, pbs[1]));
                const float2 q0 = __fmul2_rn(pv, vsa);
                const float2 q1 = __fmul2_rn(pv, vsb);
                pw0[kk / 2] = pack_h2(q0.x, q0.y);
                pw1[kk / 2] = pack_h2(q1.x, q1.y);
              }
            }
            lsum += ls2.x + ls2.y;
            tmem_st16(lane_base + 256 + c0 / 2, pw0);
            tmem_st16(lane_base + 320 + c0 / 2, pw1);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        asm volatile("bar.sync 1, %0;" ::"r"(kCThreads) : "memory");
        tc_fence_after();

        // ---- 4. O_g += P'_g . V_g ----
        if (tid == 0 && !hung && !*abort_flag) {
#pragma unroll
          for (int g = 0; g < TNG; g++)
#pragma unroll
            for (int ks = 0; ks < kKeys / 16; ks++)
              umma_ts(tm + 384 + g * 64, tm + 256 + g * 64 + 8 * ks,
                      desc_sw128(smem_u32(vc + g * 16384) + 2048 * ks), idesc_pv,
                      (j > sj || ks > 0) ? 1u : 0u);
          umma_commit(pv_bar);
        }
      }
      // the unit's last PV (the earlier ones completed under the following QK commits)
      if (j1 > sj) {
        const bool ok = !hung && !*abort_flag && mbar_wait(pv_bar, (uint32_t)((tcount - 1) & 1));
        if (!__all_sync(0xffffffffu, ok)) {
          if (!hung && lane == 0) *abort_flag = 1;
          hung = true;
        }
      }
      tc_fence_after();

      // ---- epilogue: out = (2^24 O_g + sum(p vb_g)) / l, half kh writes group kh ----
      xch[(kh * 4 + 1) * kKeys + r] = lsum;
      xch[(kh * 4 + 2) * kKeys + r] = pbs[0];
      xch[(kh * 4 + 3) * kKeys + r] = pbs[1];
      asm volatile("bar.sync 1, %0;" ::"r"(kCThreads) : "memory");
      const float lt = xch[(0 * 4 + 1) * kKeys + r] + xch[(1 * 4 + 1) * kKeys + r];
      const float pbt = xch[(0 * 4 + 2 + kh) * kKeys + r] + xch[(1 * 4 + 2 + kh) * kKeys + r];
      if (!partial) {
        const int64_t orow = ((int64_t)b * p.Hq + kvh * nrep + hh) * L + l;
        uint16_t* dst = p.out + orow * TD + kh * TGS;
        const bool have_o = !hung && j1 > sj;  // warp-uniform: TMEM loads are collective
#pragma unroll 1
        for (int c0 = 0; c0 < TGS; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(lane_base + 384 + kh * TGS + c0, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int k = 0; k < 32; k++) o[k] = 0u;
          }
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float v0 = lt > 0.0f ? fmaf(__uint_as_float(o[k]), kCodeUnitInv, pbt) / lt : 0.0f;
            const float v1 = lt > 0.0f ? fmaf(__uint_as_float(o[k + 1]), kCodeUnitInv, pbt) / lt : 0.0f;
            w[k / 2] = (uint32_t)f_to_dt<BF>(v0) | ((uint32_t)f_to_dt<BF>(v1) << 16);
          }
          if (qvalid) {
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<uint4*>(dst + c0 + 2 * k) = make_uint4(w[k], w[k + 1], w[k + 2], w[k + 3]);
          }
        }
      } else {
        // partial of a unit this CTA covers in part: row r of slot 2c (the
        // CTA's first unit) or 2c + 1 (its last) as [m, l, sum(p vb_0),
        // sum(p vb_1), O'(128)], O' = 2^-24 O (the merge kernel finishes it)
        float* srow = p.ws_o + (((size_t)blockIdx.x * 2 + (seg ? 1 : 0)) * kRows + r) * kSlotRow;
        const bool have_o = !hung && j1 > sj;  // warp-uniform: TMEM loads are collective
#pragma unroll 1
        for (int c0 = 0; c0 < TGS; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(lane_base + 384 + kh * TGS + c0, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int k = 0; k < 32; k++) o[k] = 0u;
          }
          if (qvalid) {
#pragma unroll
            for (int k = 0; k < 32; k += 4)
              *reinterpret_cast<float4*>(srow + 4 + kh * TGS + c0 + k) =
                  make_float4(__uint_as_float(o[k]) * kCodeUnitInv, __uint_as_float(o[k + 1]) * kCodeUnitInv,
                              __uint_as_float(o[k + 2]) * kCodeUnitInv, __uint_as_float(o[k + 3]) * kCodeUnitInv);
          }
        }
        if (qvalid) {
          if (kh == 0) {
            srow[0] = m_used;
            srow[1] = lt;
          }
          srow[2 + kh] = pbt;
        }
      }
      t += j1 - sj;
      sj = 0;
      seg++;
      if (++qt == nqb) {
        qt = 0;
        ++hp;
      }
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

}  // namespace

bool prefill_tc_supported(int bits, int D, int gs, int L, bool scores) {
  return bits == 8 && D == TD && gs == TGS && L > 1 && !scores;
}

int32_t launch_prefill_tc(Params& p, int B, void* ws, size_t ws_bytes, cudaStream_t st) {
  auto kern = p.bf16 ? prefill_tc_kernel<true> : prefill_tc_kernel<false>;
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  int32_t rc = kernel_setup(reinterpret_cast<const void*>(kern), kCThreads + 32, kTcSmem, dev, nullptr);
  if (rc) return rc;
  const int qrows = p.nrep * p.L;
  const int nqb = (qrows + kRows - 1) / kRows;
  // Balanced grid (one CTA per SM, equal runs of key tiles, a merge for the
  // units cut at run boundaries) unless the batch is ragged (per-sequence
  // key counts live on the device) or the caller's workspace is too small.
  int64_t ctas = 0, Th = 0;
  size_t need = kPartialOff;
  if (!p.seq_lens) {
    for (int q = 0; q < nqb; q++)
      Th += tc_block_tiles<kKeys>(q, p.N, p.L, p.nrep, p.mask_mode, p.window);
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
    KVQ_CUDA_TRY(launch_pdl(kern, dim3((unsigned)ctas), dim3(kCThreads + 32), (size_t)kTcSmem, st, p));
    auto merge = p.bf16 ? prefill_tc_merge_kernel<true, kKeys> : prefill_tc_merge_kernel<false, kKeys>;
    KVQ_CUDA_TRY(launch_pdl(merge, dim3((unsigned)ctas), dim3(kMergeThreads), 0, st, p));
    return KVQ_OK;
  }
  const dim3 grid((unsigned)nqb, (unsigned)p.Hkv, (unsigned)B);
  KVQ_CUDA_TRY(launch_pdl(kern, grid, dim3(kCThreads + 32), (size_t)kTcSmem, st, p));
  return KVQ_OK;
}

}  // namespace attn
}  // namespace kvq
