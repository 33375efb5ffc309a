// kvq_quant.cu — quantize-on-append for sm_100a.
//
// One thread owns one packed uint32 of a row (32/bits consecutive elements);
// the gs*bits/32 threads of a quantization group reduce min/max with warp
// shuffles, apply the affine rule of MLX's quantize (as restated and pinned
// by the oracle: anchor = larger-magnitude extreme, scale = anchor /
// round(anchor / s0), codes from the unrounded f32 scale, round half away
// from zero, clamp to [0, 2^bits-1]) and write their word; lane 0 of the
// group writes the dtype-rounded scale and the bias.  Divisions are IEEE
// (no fast-math) so the codes are bit-identical to the CPU restatement.
//
// One launch carries up to two jobs (the K and the V rows of an append,
// selected by blockIdx.y): on the decode path the work is a few rows and the
// launch itself is the cost.
//
// Ragged appends (RAG): batch entry b writes its first counts[b] rows at
// rows lens[b] + s of its (b, h) rows, where lens and counts are device
// arrays — the positions live on the GPU, so a captured CUDA graph appends
// at a new position on every replay.  A separate launch
// (ragged_advance_kernel) then adds counts[b] to lens[b].  An entry whose
// rows would pass the capacity is skipped by both launches and raises the
// cache's error flag.  For whole-cache conversion the kernel is
// HBM-bound: 2 B read and bits/8 + 4/gs B written per element, with 16-byte
// loads when the input rows are 16-byte aligned.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kvq_internal.h"
#include "kvq_qrule.cuh"

namespace kvq {
namespace {

struct Job {
  const uint16_t* x;
  int64_t sb, sh, ss;  // element strides of (b, h, s); d stride is 1
  uint32_t* packed;
  uint16_t* scales;
  uint16_t* biases;
  int64_t dst_bstride, dst_hstride, dst_row0;  // rows
};

struct Jobs {
  Job j[2];
  int H, S, words;
  int64_t total_rows;
  const int32_t* lens;    // ragged: device [B] first destination row per entry
  const int32_t* counts;  // ragged: device [B] rows to write per entry (nullable: S)
  int64_t cap;            // ragged: rows per (b, h)
  int* err;               // ragged: cache error flag
};

template <bool BF16>
__device__ __forceinline__ float load_f(const uint16_t* p) {
  const uint16_t v = __ldg(p);
  if (BF16) return __uint_as_float((uint32_t)v << 16);
  return __half2float(__ushort_as_half(v));
}

template <bool BF16>
__device__ __forceinline__ uint16_t store_bits(float f) {
  if (BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  return __half_as_ushort(__float2half_rn(f));
}

template <bool BF16>
__device__ __forceinline__ float word_to_f(uint32_t w, int half) {
  const uint16_t v = (uint16_t)(half ? (w >> 16) : (w & 0xffffu));
  if (BF16) return __uint_as_float((uint32_t)v << 16);
  return __half2float(__ushort_as_half(v));
}

// BITS: 4 or 8.  TPG: threads per group (gs * BITS / 32).  VEC: 16-B loads.
// RAG: ragged destination rows (lens / counts).
template <int BITS, int TPG, bool BF16, bool VEC, bool RAG = false>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const Jobs jobs) {
  // launched as a programmatic dependent (launch_pdl): let the next kernel be
  // scheduled, then wait for the previous one before reading anything
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int PER = 32 / BITS;
  constexpr float NB = (float)((1 << BITS) - 1);
  const Job& J = jobs.j[blockIdx.y];
  const int words = jobs.words;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = tid / words;
  const int word = (int)(tid - row * words);
  const bool valid = row < jobs.total_rows;
  const int64_t r = valid ? row : jobs.total_rows - 1;
  const int s = (int)(r % jobs.S);
  const int64_t bh = r / jobs.S;
  const int h = (int)(bh % jobs.H);
  const int64_t b = bh / jobs.H;
  const uint16_t* src = J.x + b * J.sb + h * J.sh + (int64_t)s * J.ss + (int64_t)word * PER;

  float w[PER];
  if (VEC) {
    if (PER == 8) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
      const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        w[2 * i] = word_to_f<BF16>(q[i], 0);
        w[2 * i + 1] = word_to_f<BF16>(q[i], 1);
      }
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(src));
      w[0] = word_to_f<BF16>(u.x, 0);
      w[1] = word_to_f<BF16>(u.x, 1);
      w[2] = word_to_f<BF16>(u.y, 0);
      w[3] = word_to_f<BF16>(u.y, 1);
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; i++) w[i] = load_f<BF16>(src + i);
  }
  float mn = w[0], mx = w[0];
#pragma unroll
  for (int i = 1; i < PER; i++) {
    mn = fminf(mn, w[i]);
    mx = fmaxf(mx, w[i]);
  }
#pragma unroll
  for (int off = 1; off < TPG; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  float scale, bias;
  quant_params(mn, mx, NB, scale, bias);
  uint32_t out = 0;
#pragma unroll
  for (int i = 0; i < PER; i++) out |= quant_code(w[i], scale, bias, NB) << (BITS * i);
  int64_t row0 = J.dst_row0;
  if (RAG) {
    const int64_t l0 = jobs.lens[b];
    const int64_t cnt = jobs.counts ? jobs.counts[b] : jobs.S;
    if (cnt < 0 || l0 < 0 || l0 + cnt > jobs.cap) {
      if (valid && s == 0 && word == 0) atomicExch(jobs.err, 1);
      return;
    }
    if (s >= cnt) return;
    row0 += l0;
  }
  if (!valid) return;
  const int64_t drow = b * J.dst_bstride + h * J.dst_hstride + row0 + s;
  J.packed[drow * words + word] = out;
  if ((word % TPG) == 0) {
    const int groups = words / TPG;
    const int g = word / TPG;
    J.scales[drow * groups + g] = store_bits<BF16>(scale);
    J.biases[drow * groups + g] = store_bits<BF16>(bias);
  }
}

// lens[b] += counts[b] (or S) after the ragged quantize launch has read
// them; entries the quantize launch skipped (past the capacity) stay put.
__global__ void ragged_advance_kernel(int32_t* __restrict__ lens, const int32_t* __restrict__ counts,
                                      int S, int B, int64_t cap) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t l0 = lens[b];
  const int64_t cnt = counts ? counts[b] : S;
  if (cnt >= 0 && l0 >= 0 && l0 + cnt <= cap) lens[b] = (int32_t)(l0 + cnt);
}

template <int BITS, int TPG, bool BF16>
int32_t dispatch_vec(bool vec, dim3 grid, cudaStream_t st, const Jobs& jobs) {
  if (jobs.lens) {
    if (vec)
      KVQ_CUDA_TRY(launch_pdl(quantize_rows_kernel<BITS, TPG, BF16, true, true>, grid, dim3(256), 0, st, jobs));
    else
      KVQ_CUDA_TRY(launch_pdl(quantize_rows_kernel<BITS, TPG, BF16, false, true>, grid, dim3(256), 0, st, jobs));
    return KVQ_OK;
  }
  if (vec)
    KVQ_CUDA_TRY(launch_pdl(quantize_rows_kernel<BITS, TPG, BF16, true>, grid, dim3(256), 0, st, jobs));
  else
    KVQ_CUDA_TRY(launch_pdl(quantize_rows_kernel<BITS, TPG, BF16, false>, grid, dim3(256), 0, st, jobs));
  return KVQ_OK;
}

template <int BITS, bool BF16>
int32_t dispatch_tpg(int tpg, bool vec, dim3 grid, cudaStream_t st, const Jobs& jobs) {
  switch (tpg) {
    case 4: return dispatch_vec<BITS, 4, BF16>(vec, grid, st, jobs);
    case 8: return dispatch_vec<BITS, 8, BF16>(vec, grid, st, jobs);
    case 16: return dispatch_vec<BITS, 16, BF16>(vec, grid, st, jobs);
    case 32: return dispatch_vec<BITS, 32, BF16>(vec, grid, st, jobs);
  }
  return fail(KVQ_ERR_ARG, "quantize: unsupported group_size/bits combination");
}

bool aligned_for(const Job& j, int per) {
  return ((uintptr_t)j.x % (per * 2) == 0) && j.sb % per == 0 && j.sh % per == 0 &&
         j.ss % per == 0;
}

int32_t launch_jobs(Jobs& jobs, int njobs, int B, RowGeom g, int dtype, cudaStream_t st) {
  jobs.total_rows = (int64_t)B * jobs.H * jobs.S;
  if (jobs.total_rows == 0) return KVQ_OK;
  jobs.words = g.words();
  const int tpg = g.gs * g.bits / 32;
  const int per = 32 / g.bits;
  const int64_t threads = jobs.total_rows * jobs.words;
  const dim3 grid((unsigned)((threads + 255) / 256), (unsigned)njobs);
  bool vec = true;
  for (int i = 0; i < njobs; i++) vec = vec && aligned_for(jobs.j[i], per);
  const bool bf = dtype == KVQ_DTYPE_BFLOAT16;
  if (g.bits == 4)
    return bf ? dispatch_tpg<4, true>(tpg, vec, grid, st, jobs)
              : dispatch_tpg<4, false>(tpg, vec, grid, st, jobs);
  return bf ? dispatch_tpg<8, true>(tpg, vec, grid, st, jobs)
            : dispatch_tpg<8, false>(tpg, vec, grid, st, jobs);
}

Job job_for(const void* x, const int64_t* strides, const TripleView& d, int64_t row0) {
  Job j;
  j.x = static_cast<const uint16_t*>(x);
  j.sb = strides[0];
  j.sh = strides[1];
  j.ss = strides[2];
  j.packed = d.packed;
  j.scales = d.scales;
  j.biases = d.biases;
  j.dst_bstride = d.batch_stride;
  j.dst_hstride = d.head_stride;
  j.dst_row0 = row0;
  return j;
}

}  // namespace

int32_t launch_append_kv(const void* k, const int64_t* k_strides, const void* v,
                         const int64_t* v_strides, int B, int H, int S, RowGeom g, int dtype,
                         TripleView dk, TripleView dv, int64_t dst_row0, cudaStream_t st) {
  Jobs jobs{};
  jobs.j[0] = job_for(k, k_strides, dk, dst_row0);
  jobs.j[1] = job_for(v, v_strides, dv, dst_row0);
  jobs.H = H;
  jobs.S = S;
  return launch_jobs(jobs, 2, B, g, dtype, st);
}

int32_t launch_append_ragged(const void* k, const int64_t* k_strides, const void* v,
                             const int64_t* v_strides, int B, int H, int S, RowGeom g, int dtype,
                             TripleView dk, TripleView dv, int64_t cap, int32_t* lens,
                             const int32_t* counts, int* err, cudaStream_t st) {
  Jobs jobs{};
  jobs.j[0] = job_for(k, k_strides, dk, 0);
  jobs.j[1] = job_for(v, v_strides, dv, 0);
  jobs.H = H;
  jobs.S = S;
  jobs.lens = lens;
  jobs.counts = counts;
  jobs.cap = cap;
  jobs.err = err;
  int32_t rc = launch_jobs(jobs, 2, B, g, dtype, st);
  if (rc) return rc;
  KVQ_CUDA_TRY(launch_pdl(ragged_advance_kernel, dim3((unsigned)((B + 127) / 128)), dim3(128), 0,
                          st, lens, counts, S, B, cap));
  return KVQ_OK;
}

int32_t launch_quantize_rows(const void* x, int64_t rows, RowGeom g, int dtype, uint32_t* packed,
                             uint16_t* scales, uint16_t* biases, cudaStream_t st) {
  if (rows > (int64_t)0x7fffffff) return fail(KVQ_ERR_ARG, "quantize: too many rows");
  // Treat the rows as [1, 1, rows, D].
  const int64_t strides[3] = {0, 0, g.D};
  TripleView d{packed, scales, biases, 0, 0};
  Jobs jobs{};
  jobs.j[0] = job_for(x, strides, d, 0);
  jobs.H = 1;
  jobs.S = (int)rows;
  return launch_jobs(jobs, 1, 1, g, dtype, st);
}

}  // namespace kvq
