// kvq_attn_b8.cu — instantiations of the attention kernel for 8-bit codes.
#include "kvq_attn_impl.cuh"

namespace kvq {
namespace attn {

template <int BITS, int D, int GS, int NT>
int32_t launch_t(Params& p, const LaunchShape& s, int B, cudaStream_t st, int* occ) {
  constexpr int RW = rows_per_warp<D, NT>();
  constexpr int ST = stages_for<BITS, D, GS, RW>();
  using SM = Smem<BITS, D, GS, NT, kWarps, RW, ST>;
  auto kern = p.bf16 ? attn_kernel<BITS, D, GS, NT, kWarps, RW, ST, true>
                     : attn_kernel<BITS, D, GS, NT, kWarps, RW, ST, false>;
  static int blocks[2][64] = {{0}};
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(KVQ_ERR_ARG, "device ordinal out of range");
  if (!blocks[p.bf16][dev]) {
    KVQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL));
    int n = 0;
    KVQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, (kWarps + 1) * 32, SM::TOTAL));
    blocks[p.bf16][dev] = n > 0 ? n : 1;
  }
  if (occ) {
    *occ = blocks[p.bf16][dev];
    return KVQ_OK;
  }
  const dim3 grid(s.nsplit, p.Hkv * s.QB, B);
  kern<<<grid, (kWarps + 1) * 32, SM::TOTAL, st>>>(p);
  KVQ_CUDA_TRY(cudaGetLastError());
  return KVQ_OK;
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
static int32_t pick_d(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st, int* occ) {
  switch (Dv) {
    case 64: return pick_gs<BITS, 64>(p, s, GSv, NT, B, st, occ);
    case 128: return pick_gs<BITS, 128>(p, s, GSv, NT, B, st, occ);
    case 256: return pick_gs<BITS, 256>(p, s, GSv, NT, B, st, occ);
  }
  return fail(KVQ_ERR_ARG, "attention: head_dim must be 64, 128 or 256");
}


int32_t dispatch_b8(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st,
                    int* occ) {
  return pick_d<8>(p, s, Dv, GSv, NT, B, st, occ);
}

}  // namespace attn
}  // namespace kvq
