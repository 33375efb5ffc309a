// kvq_noalloc.cu — decode attention that allocates no device memory.
//
// Some callers cannot have device memory allocated on their behalf:
// serving processes that hand all free device memory to their own pool at
// start-up (a cudaMalloc then fails, or takes memory the pool counts on),
// and latency-bound decode loops that must never meet the implicit device
// synchronization of a cudaMalloc.  For them kvq_sdpa_decode_noalloc runs
// the same decode kernels as kvq_sdpa_decode but keeps their scratch
// (device error flag, split tickets, split partials) in the file-scope
// array below instead of a cudaMalloc'd buffer.  When the partials of the
// full launch would not fit, the decode is spread over fewer CTAs (fewer
// partials) so that they do; shapes whose partials do not fit even with a
// single CTA are refused.
//
// The array is KVQ_NOALLOC_SCRATCH_BYTES long; every GPU that loads the
// library holds it until the process exits.  Host code cannot use the
// array's name as a device address, so the first call on each device (with
// that device current) looks the address up once with cudaGetSymbolAddress;
// make that first call before any stream capture.  Every call shares the
// array and leaves its contents behind, so each call clears the part that
// must start at zero (the split tickets) with a stream-ordered memset, and
// calls that overlap on the GPU race: issue them on one stream.  The device
// error flag at the start of the array is not cleared by a call: a bounded
// wait that timed out stays visible until kvq_check_device(NULL, ...) on
// that device reports and clears it.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "kvq_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[KVQ_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of g_decode_scratch on the current device.
int32_t scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= 64) return kvq::fail(KVQ_ERR_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || !p) return kvq::cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KVQ_OK;
}

}  // namespace

void* kvq::noalloc_scratch_if_known(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  return g_scratch_ptr[dev];
}

extern "C" int32_t kvq_sdpa_decode_noalloc(const kvq_qtensor* keys, const kvq_qtensor* values,
                                           const void* q, int32_t q_heads, float scale,
                                           const int32_t* seq_lens, void* out, void* stream) {
  using namespace kvq;
  AttnArgs a{};
  int32_t rc = make_attn_args(keys, values, q, q_heads, scale, seq_lens, a);
  if (rc) return rc;
  if (!out) return fail(KVQ_ERR_ARG, "out is NULL");
  size_t need = 0, zero_prefix = 0;
  if ((rc = decode_workspace_exact(a, &need, &zero_prefix, (size_t)KVQ_NOALLOC_SCRATCH_BYTES)))
    return rc;
  if (need > (size_t)KVQ_NOALLOC_SCRATCH_BYTES)
    return fail(KVQ_ERR_WORKSPACE,
                "kvq_sdpa_decode_noalloc: these shapes need " + std::to_string(need) +
                    " bytes of scratch, more than its fixed " +
                    std::to_string((size_t)KVQ_NOALLOC_SCRATCH_BYTES) +
                    "; use kvq_sdpa_decode with a caller workspace");
  int dev = 0;
  KVQ_CUDA_TRY(cudaGetDevice(&dev));
  void* ws = nullptr;
  if ((rc = scratch_address(dev, &ws))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Clear the tickets only: the error flag (the first kWsFlagBytes) keeps a
  // timeout raised by an earlier call until kvq_check_device reports it.
  if (zero_prefix > kWsFlagBytes)
    KVQ_CUDA_TRY(cudaMemsetAsync(static_cast<uint8_t*>(ws) + kWsFlagBytes, 0,
                                 zero_prefix - kWsFlagBytes, st));
  return launch_decode(a, out, nullptr, nullptr, nullptr, ws, (size_t)KVQ_NOALLOC_SCRATCH_BYTES,
                       st, /*fit_to_ws=*/true);
}
