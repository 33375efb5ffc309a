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
// The kernel is HBM-bound and tiny on the decode path (S = 1 row per head);
// for whole-cache conversion it reads 2 B and writes bits/8 + 4/gs B per
// element with 16-byte loads when the input rows are 16-byte aligned.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kvq_internal.h"

namespace kvq {
namespace {

constexpr float kEps = 1e-7f;  // constant-group guard shared with the oracle

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
template <int BITS, int TPG, bool BF16, bool VEC>
__global__ void __launch_bounds__(256) quantize_rows_kernel(
    const uint16_t* __restrict__ x, int64_t sb, int64_t sh, int64_t ss, int H, int S,
    int64_t total_rows, int words, uint32_t* __restrict__ packed, uint16_t* __restrict__ scales,
    uint16_t* __restrict__ biases, int64_t dst_bstride, int64_t dst_hstride, int64_t dst_row0) {
  constexpr int PER = 32 / BITS;
  constexpr float NB = (float)((1 << BITS) - 1);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = tid / words;
  const int word = (int)(tid - row * words);
  const bool valid = row < total_rows;
  const int64_t r = valid ? row : total_rows - 1;
  const int s = (int)(r % S);
  const int64_t bh = r / S;
  const int h = (int)(bh % H);
  const int64_t b = bh / H;
  const uint16_t* src = x + b * sb + h * sh + (int64_t)s * ss + (int64_t)word * PER;

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
  float s0 = (mx - mn) / NB;
  if (!(s0 >= kEps)) s0 = kEps;
  const bool neg = fabsf(mn) > fabsf(mx);
  const float anchor = neg ? mn : mx;
  s0 = neg ? s0 : -s0;
  const float q0 = roundf(anchor / s0);
  float scale, bias;
  if (q0 != 0.0f) {
    scale = anchor / q0;
    bias = anchor;
  } else {
    scale = s0;
    bias = 0.0f;
  }
  uint32_t out = 0;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    float c = roundf((w[i] - bias) / scale);
    c = fminf(fmaxf(c, 0.0f), NB);
    out |= (uint32_t)c << (BITS * i);
  }
  if (!valid) return;
  const int64_t drow = b * dst_bstride + h * dst_hstride + dst_row0 + s;
  packed[drow * words + word] = out;
  if ((word % TPG) == 0) {
    const int groups = words / TPG;
    const int g = word / TPG;
    scales[drow * groups + g] = store_bits<BF16>(scale);
    biases[drow * groups + g] = store_bits<BF16>(bias);
  }
}

template <int BITS, int TPG, bool BF16>
int32_t dispatch_vec(bool vec, dim3 grid, cudaStream_t st, const uint16_t* x, int64_t sb,
                     int64_t sh, int64_t ss, int H, int S, int64_t total, int words, TripleView d,
                     int64_t row0) {
  if (vec)
    quantize_rows_kernel<BITS, TPG, BF16, true><<<grid, 256, 0, st>>>(
        x, sb, sh, ss, H, S, total, words, d.packed, d.scales, d.biases, d.batch_stride,
        d.head_stride, row0);
  else
    quantize_rows_kernel<BITS, TPG, BF16, false><<<grid, 256, 0, st>>>(
        x, sb, sh, ss, H, S, total, words, d.packed, d.scales, d.biases, d.batch_stride,
        d.head_stride, row0);
  KVQ_CUDA_TRY(cudaGetLastError());
  return KVQ_OK;
}

template <int BITS, bool BF16>
int32_t dispatch_tpg(int tpg, bool vec, dim3 grid, cudaStream_t st, const uint16_t* x,
                     int64_t sb, int64_t sh, int64_t ss, int H, int S, int64_t total, int words,
                     TripleView d, int64_t row0) {
  switch (tpg) {
    case 2: return dispatch_vec<BITS, 2, BF16>(vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
    case 4: return dispatch_vec<BITS, 4, BF16>(vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
    case 8: return dispatch_vec<BITS, 8, BF16>(vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
    case 16: return dispatch_vec<BITS, 16, BF16>(vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
    case 32: return dispatch_vec<BITS, 32, BF16>(vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
  }
  return fail(KVQ_ERR_ARG, "quantize: unsupported group_size/bits combination");
}

int32_t launch_generic(const uint16_t* x, int64_t sb, int64_t sh, int64_t ss, int B, int H, int S,
                       RowGeom g, int dtype, TripleView d, int64_t row0, cudaStream_t st) {
  const int64_t total = (int64_t)B * H * S;
  if (total == 0) return KVQ_OK;
  const int words = g.words();
  const int tpg = g.gs * g.bits / 32;
  const int per = 32 / g.bits;
  const int64_t threads = total * words;
  const dim3 grid((unsigned)((threads + 255) / 256));
  const bool vec = ((uintptr_t)x % (per * 2) == 0) && sb % per == 0 && sh % per == 0 &&
                   ss % per == 0;
  const bool bf = dtype == KVQ_DTYPE_BFLOAT16;
  if (g.bits == 4)
    return bf ? dispatch_tpg<4, true>(tpg, vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0)
              : dispatch_tpg<4, false>(tpg, vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
  return bf ? dispatch_tpg<8, true>(tpg, vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0)
            : dispatch_tpg<8, false>(tpg, vec, grid, st, x, sb, sh, ss, H, S, total, words, d, row0);
}

}  // namespace

int32_t launch_append(const void* x, const int64_t* strides, int B, int H, int S, RowGeom g,
                      int dtype, TripleView dst, int64_t dst_row0, cudaStream_t st) {
  return launch_generic(static_cast<const uint16_t*>(x), strides[0], strides[1], strides[2], B, H,
                        S, g, dtype, dst, dst_row0, st);
}

int32_t launch_quantize_rows(const void* x, int64_t rows, RowGeom g, int dtype, uint32_t* packed,
                             uint16_t* scales, uint16_t* biases, cudaStream_t st) {
  // Treat the rows as [1, 1, rows, D]; rows may exceed int range only via S.
  if (rows > (int64_t)0x7fffffff) return fail(KVQ_ERR_ARG, "quantize: too many rows");
  TripleView d{packed, scales, biases, 0, 0};
  return launch_generic(static_cast<const uint16_t*>(x), 0, 0, g.D, 1, 1, (int)rows, g, dtype, d,
                        0, st);
}

}  // namespace kvq
