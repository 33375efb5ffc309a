// kvq_attn.cu — host side of the attention entry points: argument checks,
// kernel choice and launch shapes, workspace, the cross-device merge kernel
// and debug scores.  The kernels are in kvq_attn_impl.cuh, instantiated in
// kvq_attn_b4.cu / kvq_attn_b8.cu.
#include "kvq_attn_impl.cuh"

namespace kvq {
namespace attn {

// Merge of per-device partials (context split).
__global__ void merge_kernel(const float* __restrict__ m, const float* __restrict__ l,
                             const float* __restrict__ o, int parts, int64_t ps, int rows, int D,
                             int bf, uint16_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * D) return;
  const int r = (int)(i / D), d = (int)(i - (int64_t)r * D);
  float M = kNeg;
  for (int pp = 0; pp < parts; pp++) M = fmaxf(M, m[pp * ps + r]);
  float Ls = 0.0f, O = 0.0f;
  for (int pp = 0; pp < parts; pp++) {
    const float e = ex2((m[pp * ps + r] - M) * kLog2e);
    Ls += l[pp * ps + r] * e;
    O += o[pp * ps + (int64_t)r * D + d] * e;
  }
  out[i] = bf ? f_to_dt<true>(Ls > 0.0f ? O / Ls : 0.0f) : f_to_dt<false>(Ls > 0.0f ? O / Ls : 0.0f);
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}


// Validate and fill Params common to every attention launch.
int32_t prepare(const AttnArgs& a, int L, int mask_mode, int window, Params& p, int& NT) {
  if (a.Hkv <= 0 || a.Hq <= 0 || a.Hq % a.Hkv) return fail(KVQ_ERR_ARG, "q_heads must be a multiple of kv heads");
  const int nrep = a.Hq / a.Hkv;
  NT = nrep * L <= 8 ? 1 : 2;
  if (L == 1 && nrep > 16) return fail(KVQ_ERR_ARG, "decode: more than 16 query heads per kv head");
  if (a.bits != 4 && a.bits != 8) return fail(KVQ_ERR_ARG, "bits must be 4 or 8");
  if (a.gs != 32 && a.gs != 64 && a.gs != 128) return fail(KVQ_ERR_ARG, "group_size must be 32, 64 or 128");
  if (a.D % a.gs) return fail(KVQ_ERR_ARG, "head_dim must be a multiple of group_size");
  if (a.dtype != KVQ_DTYPE_FLOAT16 && a.dtype != KVQ_DTYPE_BFLOAT16) return fail(KVQ_ERR_ARG, "dtype must be float16 or bfloat16");
  // TMA bulk copies read whole 16-row tiles: row strides must keep every tile
  // 16-byte aligned and inside its head's rows.
  const int64_t strides[4] = {a.k.batch_stride, a.k.head_stride, a.v.batch_stride, a.v.head_stride};
  for (int i = 0; i < 4; i++)
    if (strides[i] % kTile) return fail(KVQ_ERR_ARG, "view row strides must be multiples of 16 rows");
  const uintptr_t ptrs[6] = {(uintptr_t)a.k.packed, (uintptr_t)a.k.scales, (uintptr_t)a.k.biases,
                             (uintptr_t)a.v.packed, (uintptr_t)a.v.scales, (uintptr_t)a.v.biases};
  for (int i = 0; i < 6; i++)
    if (ptrs[i] % 16) return fail(KVQ_ERR_ARG, "view base pointers must be 16-byte aligned");
  if (a.N > 0) {
    // The last tile is read whole: the rows up to the next multiple of 16
    // must exist.  Views from a kvq_cache always satisfy this.
    const int64_t need = (int64_t)(a.N + kTile - 1) / kTile * kTile;
    if (need > a.k.head_stride || need > a.v.head_stride)
      return fail(KVQ_ERR_ARG, "view head_stride must cover len rounded up to 16 rows");
  }
  p = Params{};
  p.kp = reinterpret_cast<const uint8_t*>(a.k.packed);
  p.ks = a.k.scales;
  p.kb = a.k.biases;
  p.vp = reinterpret_cast<const uint8_t*>(a.v.packed);
  p.vs = a.v.scales;
  p.vb = a.v.biases;
  p.k_bstride = a.k.batch_stride;
  p.k_hstride = a.k.head_stride;
  p.v_bstride = a.v.batch_stride;
  p.v_hstride = a.v.head_stride;
  p.q = static_cast<const uint16_t*>(a.q);
  p.seq_lens = a.seq_lens;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.nrep = nrep;
  p.N = a.N;
  p.L = L;
  p.mask_mode = mask_mode;
  p.window = window;
  p.scale = a.scale;
  p.bf16 = a.dtype == KVQ_DTYPE_BFLOAT16;
  return KVQ_OK;
}

// Kernel choice, launch shape and workspace of one attention call.
struct Plan {
  LaunchShape s;
  size_t ws_bytes;  // workspace this call needs
  int64_t tickets;  // merge tickets it uses (zero before and after the call)
};

// budget: the workspace bytes available; the balanced decode spreads over
// fewer CTAs when its partials would not fit (fewer slots), down to one.
int32_t make_plan(const AttnArgs& a, int L, int mask_mode, int window, bool scores, Params& p,
                  int& NT, Plan& pl, size_t budget = SIZE_MAX) {
  int32_t rc = prepare(a, L, mask_mode, window, p, NT);
  if (rc) return rc;
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  const int64_t units = (int64_t)a.B * a.Hkv;
  // Decode over every key of each row: the balanced single-wave kernel.
  // (its TMA copies of the query rows need a 16-byte aligned q)
  const bool bal = L == 1 && !scores && (mask_mode == 0 || window <= 0) && a.N > 0 &&
                   units > 0 && units <= kMaxTickets && (!a.seq_lens || a.B <= kBalMaxBatch) &&
                   reinterpret_cast<uintptr_t>(a.q) % 16 == 0;
  LaunchShape probe{1, 1, 1};
  probe.ctas = bal ? 1 : 0;
  int occ = 1;
  rc = a.bits == 4 ? dispatch_b4(p, probe, a.D, a.gs, NT, a.B, nullptr, &occ)
                   : dispatch_b8(p, probe, a.D, a.gs, NT, a.B, nullptr, &occ);
  if (rc) return rc;
  if (bal) {
    const int Tu = (a.N + kTile - 1) / kTile;
    auto working = [&](int blocks_per_sm) {
      int64_t C = (int64_t)num_sms(dev) * blocks_per_sm;
      C = std::min<int64_t>(C, std::max<int64_t>(1, units * Tu / kBalMinTiles));
      // the merge takes at most kMergeSlots partials of one unit
      C = std::min<int64_t>(C, kMergeSlots / kWarps - 1);
      if (budget != SIZE_MAX && budget > kPartialOff) {
        const int64_t fit = (int64_t)((budget - kPartialOff) / bal_group_bytes(NT, a.D)) - units;
        if (fit >= 1) C = std::min<int64_t>(C, fit);
      }
      return C;
    };
    int64_t C = working(occ);
    pl.s = LaunchShape{1, 1, kTile};
    // short ranges per CTA: the 16-row-slice instance (with seq_lens the
    // padded length bounds the range)
    if (a.D * NT <= 128 && units * Tu * kTile <= (int64_t)kBalSmallRows * C) {
      pl.s.small = true;
      LaunchShape probe_s = probe;
      probe_s.small = true;
      rc = a.bits == 4 ? dispatch_b4(p, probe_s, a.D, a.gs, NT, a.B, nullptr, &occ)
                       : dispatch_b8(p, probe_s, a.D, a.gs, NT, a.B, nullptr, &occ);
      if (rc) return rc;
      C = working(occ);
    }
    pl.s.ctas = (int)C;
    p.B = a.B;
    p.Tu = Tu;
    pl.tickets = 0;
  } else {
    pl.s = shape_for(a.B, a.Hkv, p.nrep, L, std::max(a.N, 1), NT, num_sms(dev) * occ);
    if (units * pl.s.QB > kMaxTickets) {  // too many merge groups: no key split
      pl.s.nsplit = 1;
      pl.s.rps = std::max(a.N, 1);
    }
    // a bounded workspace that cannot hold the split partials: no key split
    // (an unsplit launch needs only the flag and ticket prefix)
    if (budget != SIZE_MAX && ws_bytes_for(a.B, a.Hkv, pl.s, NT, a.D) > budget) {
      pl.s.nsplit = 1;
      pl.s.rps = std::max(a.N, 1);
    }
    pl.tickets = pl.s.nsplit > 1 ? units * pl.s.QB : 0;
  }
  pl.ws_bytes = ws_bytes_for(a.B, a.Hkv, pl.s, NT, a.D);
  return KVQ_OK;
}

int32_t run(const AttnArgs& a, int L, int mask_mode, int window, int mode, void* out, float* pm,
            float* pl_, float* po, void* ws, size_t ws_bytes, cudaStream_t st,
            float* scores = nullptr, bool fit_to_ws = false) {
  Params p;
  int NT = 1;
  Plan pl;
  int32_t rc = make_plan(a, L, mask_mode, window, scores != nullptr, p, NT, pl,
                         fit_to_ws ? ws_bytes : SIZE_MAX);
  if (rc) return rc;
  if (a.B == 0 || a.Hq == 0) return KVQ_OK;
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  const LaunchShape& s = pl.s;
  if (!ws) {
    ws = managed_workspace(dev, pl.ws_bytes, st, &rc);
    if (rc) return rc;
  } else if (ws_bytes < pl.ws_bytes) {
    return fail(KVQ_ERR_WORKSPACE, "workspace smaller than kvq_sdpa_decode_workspace()");
  }
  uint8_t* w = static_cast<uint8_t*>(ws);
  p.err = reinterpret_cast<int*>(w);
  if (s.ctas > 0) {
    p.ws_o = reinterpret_cast<float*>(w + kPartialOff);
  } else if (pl.tickets > 0) {
    const size_t slots = (size_t)a.B * a.Hkv * s.QB * s.nsplit * 8 * NT;
    p.counters = reinterpret_cast<unsigned*>(w + kTicketOff);
    p.ws_ml = reinterpret_cast<float*>(w + kPartialOff);
    p.ws_o = reinterpret_cast<float*>(w + kPartialOff + (slots * 2 * 4 + 255) / 256 * 256);
  }
  p.QB = s.QB;
  p.rps = s.rps;
  p.nsplit = s.nsplit;
  p.mode = mode;
  p.out = static_cast<uint16_t*>(out);
  p.pm = pm;
  p.pl = pl_;
  p.po = po;
  p.scores = scores;
  if (a.bits == 4) return dispatch_b4(p, s, a.D, a.gs, NT, a.B, st, nullptr);
  return dispatch_b8(p, s, a.D, a.gs, NT, a.B, st, nullptr);
}

}  // namespace attn

using namespace attn;

size_t decode_workspace_bytes(int B, int Hkv, int Hq, int N, int D) {
  if (Hkv <= 0 || Hq % Hkv) return 0;
  const int nrep = Hq / Hkv;
  const int NT = nrep <= 8 ? 1 : 2;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  // Upper bound over every kernel instance and both decode kernels, with
  // the largest possible residency (64 blocks per SM).
  LaunchShape s = shape_for(B, Hkv, nrep, 1, std::max(N, 1), NT, num_sms(dev) * 64);
  if ((int64_t)B * Hkv * s.QB > kMaxTickets) s.nsplit = 1;
  LaunchShape sb{1, 1, kTile};
  const int64_t units = (int64_t)B * Hkv;
  const int64_t Tu = (std::max(N, 0) + kTile - 1) / kTile;
  sb.ctas = (int)std::min<int64_t>((int64_t)num_sms(dev) * 64,
                                   std::max<int64_t>(1, units * Tu / kBalMinTiles));
  return std::max(ws_bytes_for(B, Hkv, s, NT, D), ws_bytes_for(B, Hkv, sb, NT, D));
}

int32_t decode_workspace_exact(const AttnArgs& a, size_t* bytes, size_t* zero_prefix,
                               size_t budget) {
  Params p;
  int NT = 1;
  Plan pl;
  int32_t rc = make_plan(a, 1, 0, 0, false, p, NT, pl, budget);
  if (rc) return rc;
  *bytes = pl.ws_bytes;
  *zero_prefix =
      kTicketOff + 4 * (size_t)std::min<int64_t>(std::max<int64_t>(pl.tickets, 0), kMaxTickets);
  return KVQ_OK;
}

int32_t launch_decode(const AttnArgs& a, void* out, float* pm, float* pl, float* po, void* ws,
                      size_t ws_bytes, cudaStream_t st, bool fit_to_ws) {
  return run(a, 1, 0, 0, out ? 0 : 1, out, pm, pl, po, ws, ws_bytes, st, nullptr, fit_to_ws);
}

int32_t launch_prefill(const AttnArgs& a, int L, int mask_mode, int window, void* out, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
  if (L <= 0) return fail(KVQ_ERR_ARG, "prefill: L must be positive");
  if (L > a.N) return fail(KVQ_ERR_ARG, "prefill: L exceeds the key length");
  const bool tc1 = prefill_tc_supported(a.bits, a.D, a.gs, L, false) &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const bool tc2 = !tc1 && prefill_tc2_supported(a.bits, a.D, a.gs, a.dtype, L) &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.q) % 16 == 0;
  if (tc2) {
    // warp-specialised tensor-core prefill for the shapes the first one does
    // not take: fp16, D 128, kv4, or kv8 with group 32 / 128
    Params p;
    int NT = 1;
    int32_t rc = prepare(a, L, mask_mode, window, p, NT);
    if (rc) return rc;
    if (a.B == 0 || a.Hq == 0) return KVQ_OK;
    p.out = static_cast<uint16_t*>(out);
    p.mode = 0;
    p.B = a.B;
    return launch_prefill_tc2(p, a.B, a.bits, a.gs, ws, ws_bytes, st);
  }
  if (tc1) {
    // tensor-core (tcgen05) prefill; its workspace holds the error flag and,
    // for the balanced grid, the partials of units split between CTAs
    Params p;
    int NT = 1;
    int32_t rc = prepare(a, L, mask_mode, window, p, NT);
    if (rc) return rc;
    if (a.B == 0 || a.Hq == 0) return KVQ_OK;
    p.out = static_cast<uint16_t*>(out);
    p.mode = 0;
    p.B = a.B;
    return launch_prefill_tc(p, a.B, ws, ws_bytes, st);
  }
  return run(a, L, mask_mode, window, 0, out, nullptr, nullptr, nullptr, ws, ws_bytes, st);
}

int32_t launch_merge(const float* m, const float* l, const float* o, int parts, int64_t pstride,
                     int rows, int D, int dtype, void* out, cudaStream_t st) {
  const int64_t n = (int64_t)rows * D;
  if (n == 0) return KVQ_OK;
  merge_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      m, l, o, parts, pstride, rows, D, dtype == KVQ_DTYPE_BFLOAT16, static_cast<uint16_t*>(out));
  KVQ_CUDA_TRY(cudaGetLastError());
  return KVQ_OK;
}

int32_t launch_debug_scores(const AttnArgs& a, int L, int mask_mode, int window, float* scores,
                            cudaStream_t st) {
  if (L <= 0 || L > a.N) return fail(KVQ_ERR_ARG, "debug scores: bad L");
  const int64_t n = (int64_t)a.B * a.Hq * L * a.N;
  if (n == 0) return KVQ_OK;
  fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(scores, n, -INFINITY);
  KVQ_CUDA_TRY(cudaGetLastError());
  void* tmp = nullptr;
  const size_t ob = (size_t)a.B * a.Hq * L * a.D * 2;
  KVQ_CUDA_TRY(cudaMallocAsync(&tmp, ob, st));
  const int32_t rc = run(a, L, mask_mode, window, 0, tmp, nullptr, nullptr, nullptr, nullptr, 0,
                         st, scores);
  cudaError_t e = cudaFreeAsync(tmp, st);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
  return KVQ_OK;
}

}  // namespace kvq
