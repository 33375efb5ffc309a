// kvq_attn_b4.cu — instantiations of the attention kernels for 4-bit codes.
#include "kvq_attn_impl.cuh"

namespace kvq {
namespace attn {

int32_t dispatch_b4(Params& p, const LaunchShape& s, int Dv, int GSv, int NT, int B, cudaStream_t st,
                    int* occ) {
  return pick_d<4>(p, s, Dv, GSv, NT, B, st, occ);
}

}  // namespace attn
}  // namespace kvq
