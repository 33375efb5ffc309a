// kvq_peer.cu — the exchange step of a context split across the GPUs of one
// node, over peer memory (CUDA IPC mappings, NVLink), with no NCCL call.
//
// A context split decodes one long sequence whose key range is cut into
// contiguous pieces, one per rank (one process per GPU).  Every rank
// computes log-sum-exp partials (m, l, o) of its piece for all query rows
// (kvq_sdpa_decode_partial, packed as [m rows | l rows | o rows*D]); this
// file moves those partials to every rank and merges them there.
//
// Each rank owns one exchange buffer in its own device memory:
//   header (256 B): [0] error flag, [4] epoch, [8] CTA ticket,
//                   [64 + 4r] arrival flag of rank r;
//   data: 2 parities x nranks slots of `slot` floats (rows*(D+2) rounded up
//         to a multiple of 64 floats).
// The buffers are exported with cudaIpcGetMemHandle and opened by every
// other rank (cudaIpcOpenMemHandle), so rank r can store into rank k's
// buffer directly.
//
// exchange_merge_kernel, one launch per step, grid = nranks CTAs:
//   * every CTA reads the step's epoch e = epoch + 1 (parity e & 1);
//   * CTA t copies this rank's packed partial into slot [parity][rank] of
//     rank t's buffer with plain 16-byte stores over NVLink and, after a
//     block barrier, sets rank t's arrival flag [rank] to e with one
//     release store at system scope;
//   * every CTA then waits (acquire loads, bounded: 2 s of %globaltimer,
//     after which it raises the error flag) until all nranks arrival flags
//     of its own buffer reach e, and merges rows [t*rows/n, (t+1)*rows/n)
//     of the nranks slots in rank order, four columns per thread with every
//     rank's loads in flight together — the same sums in the same order on
//     every rank, so all ranks produce identical outputs;
//   * the last CTA to finish (ticket) stores epoch = e.
// Two parities make the buffers reusable without a second handshake: a
// rank stores parity p of step e + 2 only after it has seen every rank's
// flag of step e + 1, which a rank raises only after its step-e merge has
// finished (kernels of one stream run in order).
// The epoch and flags live in device memory, so the step can be recorded
// once in a CUDA graph and replayed.  No TMA and no multicast is used: peer
// memory is touched only by plain loads and stores.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "kvq_internal.h"

namespace kvq {
namespace peer {

constexpr int kMaxRanks = 48;
constexpr int kHeader = 256;              // bytes before the data slots
constexpr int kFlagOff = 64;              // arrival flags (u32 per rank)
constexpr int kThreads = 512;
constexpr long long kWaitPolls = 1ll << 30;
constexpr unsigned long long kWaitNs = 2000000000ull;

struct Ptrs {
  uint8_t* buf[kMaxRanks];  // every rank's exchange buffer, as mapped here
};

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <bool BF>
__device__ __forceinline__ uint16_t to_dt(float f) {
  if constexpr (BF) {
    const __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<const uint16_t*>(&h);
  } else {
    const __half h = __float2half_rn(f);
    return *reinterpret_cast<const uint16_t*>(&h);
  }
}

// Merge of one float4 of output columns (row r, columns 4c..4c+3) over
// the NR slots at `base` (slot stride `slot` floats), in slot order.  All
// loads are issued before any arithmetic that needs them.
template <int NR, bool BF>
__device__ __forceinline__ void merge4(const float* base, int64_t slot, int rows, int D, int r,
                                       int c, int nr, uint16_t* out) {
  float m[NR], l[NR];
  float4 o[NR];
#pragma unroll
  for (int pp = 0; pp < NR; pp++) {
    if (pp < nr) {
      const float* sp = base + pp * slot;
      m[pp] = __ldcg(sp + r);
      l[pp] = __ldcg(sp + rows + r);
      o[pp] = __ldcg(reinterpret_cast<const float4*>(sp + 2 * rows + (int64_t)r * D) + c);
    } else {
      m[pp] = -1.0e30f;
      l[pp] = 0.0f;
      o[pp] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  }
  float M = -1.0e30f;
#pragma unroll
  for (int pp = 0; pp < NR; pp++) M = fmaxf(M, m[pp]);
  float Ls = 0.0f;
  float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int pp = 0; pp < NR; pp++) {
    const float w = exp2f((m[pp] - M) * 1.4426950408889634f);
    Ls = fmaf(l[pp], w, Ls);
    O.x = fmaf(o[pp].x, w, O.x);
    O.y = fmaf(o[pp].y, w, O.y);
    O.z = fmaf(o[pp].z, w, O.z);
    O.w = fmaf(o[pp].w, w, O.w);
  }
  const float inv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
  uint2 v;
  v.x = (uint32_t)to_dt<BF>(O.x * inv) | ((uint32_t)to_dt<BF>(O.y * inv) << 16);
  v.y = (uint32_t)to_dt<BF>(O.z * inv) | ((uint32_t)to_dt<BF>(O.w * inv) << 16);
  *reinterpret_cast<uint2*>(out + (int64_t)r * D + 4 * c) = v;
}

template <bool BF>
__global__ void __launch_bounds__(kThreads) exchange_merge_kernel(const Ptrs ptrs, int nranks,
                                                                  int rank, int rows, int D,
                                                                  int64_t slot,
                                                                  const float* __restrict__ local,
                                                                  uint16_t* __restrict__ out) {
  __shared__ unsigned s_epoch;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Everything below touches memory the previous kernels of the stream
  // (the partial decode, the previous exchange) wrote.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x, t = blockIdx.x;
  uint8_t* mine = ptrs.buf[rank];
  unsigned* hdr = reinterpret_cast<unsigned*>(mine);
  if (tid == 0) s_epoch = *reinterpret_cast<volatile unsigned*>(hdr + 1) + 1u;
  __syncthreads();
  const unsigned e = s_epoch;
  const int64_t par = e & 1u;
  const int64_t P = (int64_t)rows * (D + 2);  // floats of one partial set

  // ---- publish: this rank's partial into slot [par][rank] of rank t ----
  {
    float* dst = reinterpret_cast<float*>(ptrs.buf[t] + kHeader) + (par * nranks + rank) * slot;
    const bool vec = (reinterpret_cast<uintptr_t>(local) & 15) == 0;
    const int64_t n4 = vec ? P / 4 : 0;
    for (int64_t k = tid; k < n4; k += kThreads)
      reinterpret_cast<float4*>(dst)[k] = __ldg(reinterpret_cast<const float4*>(local) + k);
    for (int64_t k = n4 * 4 + tid; k < P; k += kThreads) dst[k] = __ldg(local + k);
    // The barrier orders every thread's stores before thread 0's release
    // store at system scope, which makes them visible to the rank that
    // acquires the flag.
    __syncthreads();
    if (tid == 0)
      st_release_sys(reinterpret_cast<unsigned*>(ptrs.buf[t] + kFlagOff) + rank, e);
  }

  // ---- wait for every rank's partial of this step in this rank's buffer ----
  if (tid < nranks) {
    const unsigned* f = reinterpret_cast<const unsigned*>(mine + kFlagOff) + tid;
    const unsigned long long t0 = now_ns();
    long long polls = 0;
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      if (++polls > kWaitPolls || ((polls & 255) == 0 && now_ns() - t0 > kWaitNs)) {
        atomicExch(reinterpret_cast<int*>(hdr), 1);
        break;
      }
    }
  }
  __syncthreads();

  // ---- merge rows [r0, r1), four columns per thread, in rank order ----
  const int r0 = (int)((int64_t)t * rows / nranks), r1 = (int)((int64_t)(t + 1) * rows / nranks);
  const float* base = reinterpret_cast<const float*>(mine + kHeader) + par * nranks * slot;
  const int D4 = D / 4;
  if ((rows & 1) == 0 && (D & 3) == 0 && nranks <= 8) {  // float4 columns stay 16-byte aligned
    for (int64_t i = (int64_t)r0 * D4 + tid; i < (int64_t)r1 * D4; i += kThreads) {
      const int r = (int)(i / D4), c = (int)(i - (int64_t)r * D4);
      if (nranks <= 2)
        merge4<2, BF>(base, slot, rows, D, r, c, nranks, out);
      else if (nranks <= 4)
        merge4<4, BF>(base, slot, rows, D, r, c, nranks, out);
      else
        merge4<8, BF>(base, slot, rows, D, r, c, nranks, out);
    }
  } else {
    for (int64_t i = (int64_t)r0 * D + tid; i < (int64_t)r1 * D; i += kThreads) {
      const int r = (int)(i / D), d = (int)(i - (int64_t)r * D);
      float M = -1.0e30f;
      for (int pp = 0; pp < nranks; pp++) M = fmaxf(M, __ldcg(base + pp * slot + r));
      float Ls = 0.0f, O = 0.0f;
      for (int pp = 0; pp < nranks; pp++) {
        const float* sp = base + pp * slot;
        const float w = exp2f((__ldcg(sp + r) - M) * 1.4426950408889634f);
        Ls = fmaf(__ldcg(sp + rows + r), w, Ls);
        O = fmaf(__ldcg(sp + 2 * rows + (int64_t)r * D + d), w, O);
      }
      out[i] = to_dt<BF>(Ls > 0.0f ? O / Ls : 0.0f);
    }
  }

  // ---- the last CTA to finish advances the epoch ----
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned ticket = atomicAdd(hdr + 2, 1u);
    if (ticket == (unsigned)nranks - 1) {
      hdr[2] = 0u;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(hdr + 1) = e;
    }
  }
}

}  // namespace peer
}  // namespace kvq

using namespace kvq;
using namespace kvq::peer;

struct kvq_peer_group {
  int rank = 0, nranks = 0, rows = 0, D = 0, device = 0;
  int64_t slot = 0;        // floats per slot
  size_t bytes = 0;        // exchange buffer bytes
  void* local = nullptr;   // this rank's buffer
  Ptrs ptrs{};
  std::vector<void*> opened;  // peer mappings to close
  bool connected = false;
};

extern "C" {

int32_t kvq_peer_group_create(int32_t rank, int32_t nranks, int32_t rows, int32_t head_dim,
                              void* handle_out, kvq_peer_group** out) {
  if (!out || !handle_out) return fail(KVQ_ERR_ARG, "NULL argument");
  *out = nullptr;
  if (nranks < 1 || nranks > kMaxRanks) return fail(KVQ_ERR_ARG, "nranks must be in [1, 48]");
  if (rank < 0 || rank >= nranks) return fail(KVQ_ERR_ARG, "rank out of range");
  if (rows <= 0 || head_dim <= 0) return fail(KVQ_ERR_ARG, "rows and head_dim must be positive");
  kvq_peer_group* g = new kvq_peer_group();
  g->rank = rank;
  g->nranks = nranks;
  g->rows = rows;
  g->D = head_dim;
  g->slot = ((int64_t)rows * (head_dim + 2) + 63) / 64 * 64;
  g->bytes = kHeader + (size_t)2 * nranks * g->slot * sizeof(float);
  cudaError_t e = cudaGetDevice(&g->device);
  if (e == cudaSuccess) e = cudaMalloc(&g->local, g->bytes);
  if (e == cudaSuccess) e = cudaMemset(g->local, 0, g->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
  if (e != cudaSuccess) {
    if (g->local) cudaFree(g->local);
    delete g;
    return cuda_fail(e, "kvq_peer_group_create");
  }
  std::memcpy(handle_out, &h, sizeof(h));
  g->ptrs.buf[rank] = static_cast<uint8_t*>(g->local);
  *out = g;
  return KVQ_OK;
}

int32_t kvq_peer_group_connect(kvq_peer_group* g, const void* handles) {
  if (!g || !handles) return fail(KVQ_ERR_ARG, "NULL argument");
  if (g->connected) return fail(KVQ_ERR_STATE, "peer group already connected");
  const uint8_t* hs = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < g->nranks; r++) {
    if (r == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (void* q : g->opened) cudaIpcCloseMemHandle(q);
      g->opened.clear();
      return cuda_fail(e, "cudaIpcOpenMemHandle(peer exchange buffer)");
    }
    g->opened.push_back(p);
    g->ptrs.buf[r] = static_cast<uint8_t*>(p);
  }
  g->connected = true;
  return KVQ_OK;
}

int32_t kvq_peer_exchange_merge(kvq_peer_group* g, const float* packed, int32_t dtype, void* out,
                                void* stream) {
  if (!g || !packed || !out) return fail(KVQ_ERR_ARG, "NULL argument");
  if (!g->connected && g->nranks > 1) return fail(KVQ_ERR_STATE, "peer group not connected");
  if (dtype != KVQ_DTYPE_FLOAT16 && dtype != KVQ_DTYPE_BFLOAT16) return fail(KVQ_ERR_ARG, "bad dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto kern = dtype == KVQ_DTYPE_BFLOAT16 ? exchange_merge_kernel<true> : exchange_merge_kernel<false>;
  KVQ_CUDA_TRY(launch_pdl(kern, dim3((unsigned)g->nranks), dim3(kThreads), 0, st, g->ptrs,
                          g->nranks, g->rank, g->rows, g->D, g->slot, packed,
                          static_cast<uint16_t*>(out)));
  return KVQ_OK;
}

int32_t kvq_peer_group_check(kvq_peer_group* g, void* stream) {
  if (!g) return fail(KVQ_ERR_ARG, "NULL argument");
  KVQ_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int flag = 0;
  KVQ_CUDA_TRY(cudaMemcpy(&flag, g->local, sizeof(int), cudaMemcpyDeviceToHost));
  if (flag) {
    const int zero = 0;
    KVQ_CUDA_TRY(cudaMemcpy(g->local, &zero, sizeof(int), cudaMemcpyHostToDevice));
    return fail(KVQ_ERR_CUDA, "peer exchange: a rank's partials did not arrive within 2 s");
  }
  return KVQ_OK;
}

int32_t kvq_peer_group_free(kvq_peer_group* g) {
  if (!g) return KVQ_OK;
  int32_t rc = KVQ_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != g->device) cudaSetDevice(g->device);
  cudaError_t e = cudaDeviceSynchronize();
  for (void* p : g->opened) {
    const cudaError_t e2 = cudaIpcCloseMemHandle(p);
    if (e == cudaSuccess) e = e2;
  }
  if (g->local) {
    const cudaError_t e2 = cudaFree(g->local);
    if (e == cudaSuccess) e = e2;
  }
  if (e != cudaSuccess) rc = cuda_fail(e, "kvq_peer_group_free");
  if (prev >= 0 && prev != g->device) cudaSetDevice(prev);
  delete g;
  return rc;
}

}  // extern "C"
