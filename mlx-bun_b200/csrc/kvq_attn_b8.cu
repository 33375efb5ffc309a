// kvq_attn_b8.cu — instantiations of the attention kernels for 8-bit codes.
#include "kvq_attn_impl.cuh"

namespace kvq {
namespace attn {

int32_t dispatch_b8(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st,
                    int* occ) {
  return pick_d<8>(p, s, Dv, GSv, NT, B, st, occ);
}

}  // namespace attn
}  // namespace kvq
