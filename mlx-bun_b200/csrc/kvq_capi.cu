// kvq_capi.cu — the C ABI of libkvq: cache state machines, argument checks,
// error reporting and the entry points declared in include/kvq.h.
//
// The two cache state machines restate mlx-bun's TypeScript classes
// (src/model/gemma4-base.ts) on device buffers:
//   * growing QuantizedKVCache (:419-598): capacity grows by
//     ceil(S/256)*256 rows when prev + S exceeds it, after trimming to prev
//     if prev is not 256-aligned; rows [prev, prev+S) take the new codes;
//     attention sees rows [0, offset).
//   * RotatingQuantizedKVCache (:932-1261), keep = 0: S == 1 writes in
//     place at the ring index (growing by min(256, max_size - offset) until
//     the window is full, dropping the oldest rows when the buffer is
//     oversize, rotating at max_size); S > 1 re-lays the ring out in
//     temporal order, drops rows beyond max_size - 1 and appends the S new
//     rows; attention sees rows [0, offset) before the window fills and the
//     whole buffer after.
// The reference's buffer length (keys.packed.shape[2]) is `seq_len`; the
// physical row capacity per head (`cap`, a multiple of 16) may exceed it so
// that growth inside the reservation costs no copy.  Every physical change
// of layout (growth beyond cap, front trim, temporal re-layout) is a
// stream-ordered copy into a fresh allocation.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "kvq_internal.h"

namespace kvq {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
  std::string m = std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e);
  g_last_error = m;
  return e == cudaErrorMemoryAllocation ? KVQ_ERR_OOM : KVQ_ERR_CUDA;
}

// ------------------------------------------------ library-managed scratch --

// One buffer per device, grown on demand.  A larger shape gets a new,
// larger buffer; the old one is never freed, because work already queued
// or recorded in a CUDA graph may still use it (each replay of a captured
// graph reads the pointer it was captured with).  Sizes at least double on
// each growth, so the retired buffers together stay below the live one.
struct ManagedWs {
  void* ptr = nullptr;
  size_t bytes = 0;
  std::vector<void*> retired;
};
static std::mutex g_ws_mu;
static ManagedWs g_ws[64];

void* managed_workspace(int device, size_t bytes, cudaStream_t st, int32_t* status) {
  *status = KVQ_OK;
  if (device < 0 || device >= 64) {
    *status = fail(KVQ_ERR_ARG, "device ordinal out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_ws_mu);
  ManagedWs& w = g_ws[device];
  if (w.bytes >= bytes && w.ptr) return w.ptr;
  const size_t nb = std::max({bytes, (size_t)1 << 20, 2 * w.bytes});
  void* np = nullptr;
  cudaError_t e = cudaMalloc(&np, nb);
  if (e != cudaSuccess) {
    *status = cuda_fail(e, "cudaMalloc(workspace)");
    return nullptr;
  }
  // Zero it on the calling stream and wait: the buffer is shared by every
  // stream of the device, so it must be clean before this call returns.
  e = cudaMemsetAsync(np, 0, nb, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    cudaFree(np);
    *status = cuda_fail(e, "zeroing the workspace");
    return nullptr;
  }
  if (w.ptr) w.retired.push_back(w.ptr);
  w.ptr = np;
  w.bytes = nb;
  return w.ptr;
}

// Every buffer of `device` whose error flag a kernel may have raised: the
// live workspace and the retired ones that captured graphs may still use.
static std::vector<void*> managed_ptrs(int device) {
  std::vector<void*> v;
  if (device < 0 || device >= 64) return v;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  if (g_ws[device].ptr) v.push_back(g_ws[device].ptr);
  v.insert(v.end(), g_ws[device].retired.begin(), g_ws[device].retired.end());
  return v;
}

// ------------------------------------------ per-device kernel attributes --

struct KernelKey {
  const void* kern;
  int dev, threads, smem;
  bool operator<(const KernelKey& o) const {
    if (kern != o.kern) return kern < o.kern;
    if (dev != o.dev) return dev < o.dev;
    if (threads != o.threads) return threads < o.threads;
    return smem < o.smem;
  }
};
static std::mutex g_kern_mu;
static std::map<KernelKey, int> g_kern_blocks;

int32_t kernel_setup(const void* kern, int threads, int smem, int dev, int* blocks_per_sm) {
  std::lock_guard<std::mutex> lk(g_kern_mu);
  const KernelKey key{kern, dev, threads, smem};
  auto it = g_kern_blocks.find(key);
  if (it == g_kern_blocks.end()) {
    // the attribute is per device: set it with `dev` current
    KVQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int n = 0;
    KVQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, (size_t)smem));
    it = g_kern_blocks.emplace(key, n > 0 ? n : 1).first;
  }
  if (blocks_per_sm) *blocks_per_sm = it->second;
  return KVQ_OK;
}

}  // namespace kvq

using namespace kvq;

// ------------------------------------------------------------ the cache --

struct kvq_cache {
  kvq_desc d{};
  int64_t offset = 0;
  int64_t ring_idx = 0;
  int64_t seq_len = 0;  // reference buffer length; valid when allocated
  bool allocated = false;
  int64_t cap = 0;      // physical rows per head
  void* base = nullptr; // one allocation holding the six components
  size_t bytes = 0;
  TripleView k{}, v{};
  int* status = nullptr;  // device error flag (ragged append past the capacity)

  int64_t words() const { return (int64_t)d.head_dim * d.bits / 32; }
  int64_t groups() const { return (int64_t)d.head_dim / d.group_size; }
  int64_t bh() const { return (int64_t)d.batch * d.kv_heads; }
  bool ring() const { return d.max_size > 0; }
};

namespace {

struct Layout {
  size_t off[6];
  size_t status;  // 256-byte block after the six components: the cache's error flag
  size_t total;
};

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

Layout layout_for(const kvq_cache* c, int64_t cap) {
  Layout L{};
  const size_t rows = (size_t)c->bh() * (size_t)cap;
  const size_t sz[6] = {rows * c->words() * 4, rows * c->groups() * 2, rows * c->groups() * 2,
                        rows * c->words() * 4, rows * c->groups() * 2, rows * c->groups() * 2};
  size_t o = 0;
  for (int i = 0; i < 6; i++) {
    L.off[i] = o;
    o += align256(sz[i]);
  }
  L.status = o;
  L.total = o + 256;
  return L;
}

void bind_views(kvq_cache* c, void* base, int64_t cap) {
  const Layout L = layout_for(c, cap);
  uint8_t* p = static_cast<uint8_t*>(base);
  const int64_t hs = cap, bs = cap * c->d.kv_heads;
  c->status = reinterpret_cast<int*>(p + L.status);
  c->k = TripleView{reinterpret_cast<uint32_t*>(p + L.off[0]),
                    reinterpret_cast<uint16_t*>(p + L.off[1]),
                    reinterpret_cast<uint16_t*>(p + L.off[2]), bs, hs};
  c->v = TripleView{reinterpret_cast<uint32_t*>(p + L.off[3]),
                    reinterpret_cast<uint16_t*>(p + L.off[4]),
                    reinterpret_cast<uint16_t*>(p + L.off[5]), bs, hs};
}

// Row bytes of the six components, in layout order.
void row_bytes(const kvq_cache* c, size_t rb[6]) {
  rb[0] = rb[3] = (size_t)c->words() * 4;
  rb[1] = rb[2] = rb[4] = rb[5] = (size_t)c->groups() * 2;
}

void* comp_ptr(const kvq_cache* c, int i) {
  switch (i) {
    case 0: return c->k.packed;
    case 1: return c->k.scales;
    case 2: return c->k.biases;
    case 3: return c->v.packed;
    case 4: return c->v.scales;
    default: return c->v.biases;
  }
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// One segment of rows to carry into a new allocation.
struct Seg {
  int64_t src_row, dst_row, rows;
};

// Allocate a zeroed buffer of `cap` rows per head, copy `segs` from the old
// buffer (if any), then switch to it.  Stream ordered.
int32_t relayout(kvq_cache* c, int64_t cap, const std::vector<Seg>& segs, cudaStream_t st) {
  const Layout L = layout_for(c, cap);
  void* nb = nullptr;
  KVQ_CUDA_TRY(cudaMallocAsync(&nb, L.total, st));
  KVQ_CUDA_TRY(cudaMemsetAsync(nb, 0, L.total, st));
  kvq_cache tmp = *c;
  bind_views(&tmp, nb, cap);
  size_t rb[6];
  row_bytes(c, rb);
  if (c->base) {
    for (const Seg& s : segs) {
      if (s.rows <= 0) continue;
      for (int i = 0; i < 6; i++) {
        const uint8_t* src = static_cast<const uint8_t*>(comp_ptr(c, i)) + s.src_row * rb[i];
        uint8_t* dst = static_cast<uint8_t*>(comp_ptr(&tmp, i)) + s.dst_row * rb[i];
        KVQ_CUDA_TRY(cudaMemcpy2DAsync(dst, cap * rb[i], src, c->cap * rb[i], s.rows * rb[i],
                                       (size_t)c->bh(), cudaMemcpyDeviceToDevice, st));
      }
    }
    KVQ_CUDA_TRY(cudaFreeAsync(c->base, st));
  }
  c->base = nb;
  c->bytes = L.total;
  c->cap = cap;
  bind_views(c, nb, cap);
  return KVQ_OK;
}

// Zero rows [r0, r1) of every head (the reference's appended zeros).
int32_t zero_rows(kvq_cache* c, int64_t r0, int64_t r1, cudaStream_t st) {
  if (r1 <= r0) return KVQ_OK;
  size_t rb[6];
  row_bytes(c, rb);
  for (int i = 0; i < 6; i++) {
    uint8_t* p = static_cast<uint8_t*>(comp_ptr(c, i)) + r0 * rb[i];
    KVQ_CUDA_TRY(cudaMemset2DAsync(p, c->cap * rb[i], 0, (r1 - r0) * rb[i], (size_t)c->bh(), st));
  }
  return KVQ_OK;
}

// Make the logical buffer `new_len` rows long keeping rows [0, keep) and
// zeroing [keep, new_len) (concat of zeros after a trim, :458-476, :1031-1055).
int32_t grow_to(kvq_cache* c, int64_t keep, int64_t new_len, cudaStream_t st) {
  if (c->base && new_len <= c->cap) return zero_rows(c, keep, new_len, st);
  int64_t cap = std::max<int64_t>(new_len, c->d.reserve_rows);
  if (c->ring()) cap = std::max<int64_t>(cap, c->d.max_size);
  cap = round_up(cap, c->ring() ? 16 : 256);
  std::vector<Seg> segs;
  if (c->allocated && keep > 0) segs.push_back({0, 0, keep});
  return relayout(c, cap, segs, st);
}

int32_t quantize_into(kvq_cache* c, const void* k, const void* v, int S, const int64_t* ks,
                      const int64_t* vs, int64_t dst_row, cudaStream_t st) {
  RowGeom g{c->d.head_dim, c->d.bits, c->d.group_size};
  return launch_append_kv(k, ks, v, vs, c->d.batch, c->d.kv_heads, S, g, c->d.dtype, c->k, c->v,
                          dst_row, st);
}

int32_t check_desc(const kvq_desc* d) {
  if (!d) return fail(KVQ_ERR_ARG, "desc is NULL");
  if (d->batch <= 0 || d->kv_heads <= 0) return fail(KVQ_ERR_ARG, "batch and kv_heads must be positive");
  if (d->bits != 4 && d->bits != 8) return fail(KVQ_ERR_ARG, "bits must be 4 or 8");
  if (d->group_size != 32 && d->group_size != 64 && d->group_size != 128)
    return fail(KVQ_ERR_ARG, "group_size must be 32, 64 or 128");
  if (d->head_dim <= 0 || d->head_dim % d->group_size)
    return fail(KVQ_ERR_ARG, "head_dim must be a positive multiple of group_size");
  if (d->dtype != KVQ_DTYPE_FLOAT16 && d->dtype != KVQ_DTYPE_BFLOAT16)
    return fail(KVQ_ERR_ARG, "dtype must be KVQ_DTYPE_FLOAT16 or KVQ_DTYPE_BFLOAT16");
  if (d->max_size < 0 || d->reserve_rows < 0) return fail(KVQ_ERR_ARG, "max_size / reserve_rows must be >= 0");
  return KVQ_OK;
}

int32_t check_qt(const kvq_qtensor* t, const char* name) {
  if (!t) return fail(KVQ_ERR_ARG, std::string(name) + " is NULL");
  if (!t->packed || !t->scales || !t->biases) return fail(KVQ_ERR_ARG, std::string(name) + ": NULL component pointer");
  if (t->batch <= 0 || t->heads <= 0 || t->len < 0) return fail(KVQ_ERR_ARG, std::string(name) + ": bad shape");
  return KVQ_OK;
}

struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

namespace kvq {

int32_t make_attn_args(const kvq_qtensor* k, const kvq_qtensor* v, const void* q, int32_t q_heads,
                  float scale, const int32_t* seq_lens, AttnArgs& a) {
  int32_t rc = check_qt(k, "keys");
  if (rc) return rc;
  if ((rc = check_qt(v, "values"))) return rc;
  if (!q) return fail(KVQ_ERR_ARG, "q is NULL");
  if (k->batch != v->batch || k->heads != v->heads || k->len != v->len ||
      k->head_dim != v->head_dim || k->bits != v->bits || k->group_size != v->group_size ||
      k->dtype != v->dtype)
    return fail(KVQ_ERR_ARG, "keys and values disagree in shape or quantization");
  if (q_heads <= 0 || q_heads % k->heads) return fail(KVQ_ERR_ARG, "q_heads must be a positive multiple of kv heads");
  a.k = TripleView{static_cast<uint32_t*>(k->packed), static_cast<uint16_t*>(k->scales),
                   static_cast<uint16_t*>(k->biases), k->batch_stride, k->head_stride};
  a.v = TripleView{static_cast<uint32_t*>(v->packed), static_cast<uint16_t*>(v->scales),
                   static_cast<uint16_t*>(v->biases), v->batch_stride, v->head_stride};
  a.B = k->batch;
  a.Hkv = k->heads;
  a.Hq = q_heads;
  a.N = k->len;
  a.D = k->head_dim;
  a.bits = k->bits;
  a.gs = k->group_size;
  a.dtype = k->dtype;
  a.scale = scale;
  a.q = q;
  a.seq_lens = seq_lens;
  return KVQ_OK;
}

}  // namespace kvq

namespace {

// A cache of `rows` rows per (batch, head) holding the given state: zeroed
// storage of at least `rows` rows, offset / ring index / buffer length set.
int32_t adopt_state(const kvq_desc* desc, int32_t rows, int64_t offset, int64_t ring_idx,
                    cudaStream_t st, kvq_cache** out) {
  int32_t rc = check_desc(desc);
  if (rc) return rc;
  if (rows < 0 || offset < 0) return fail(KVQ_ERR_ARG, "rows and offset must be >= 0");
  if (desc->max_size == 0 && offset > rows)
    return fail(KVQ_ERR_ARG, "growing cache: offset exceeds the buffer rows");
  if (desc->max_size > 0 && (ring_idx < 0 || ring_idx > rows))
    return fail(KVQ_ERR_ARG, "rotating cache: ring_idx must lie in [0, rows]");
  kvq_cache* c = new kvq_cache();
  c->d = *desc;
  if (rows > 0) {
    int64_t cap = std::max<int64_t>({(int64_t)rows, desc->reserve_rows,
                                     c->ring() ? (int64_t)desc->max_size : 0});
    cap = round_up(cap, c->ring() ? 16 : 256);
    if ((rc = relayout(c, cap, {}, st))) {
      delete c;
      return rc;
    }
    c->allocated = true;
    c->seq_len = rows;
  }
  c->offset = offset;
  c->ring_idx = c->ring() ? ring_idx : offset;
  *out = c;
  return KVQ_OK;
}

}  // namespace

namespace {

// The reference's update state machine for S new rows per (batch, head):
// growth, ring rotation, temporal re-layout; `write(dst_row)` fills rows
// [dst_row, dst_row + S) of every (batch, head) once the layout is ready,
// then the host state advances.  The caller selects the device.
int32_t append_rows(kvq_cache* c, int32_t S, cudaStream_t st,
                    const std::function<int32_t(int64_t)>& write) {
  int32_t rc = KVQ_OK;

  if (!c->ring()) {
    // QuantizedKVCache.updateAndFetchQuantized (:452-507)
    const int64_t prev = c->offset;
    if (!c->allocated || prev + S > c->seq_len) {
      const int64_t new_steps = (256 + (int64_t)S - 1) / 256 * 256;
      const int64_t keep = c->allocated ? ((prev % 256 != 0) ? prev : c->seq_len) : 0;
      if ((rc = grow_to(c, keep, keep + new_steps, st))) return rc;
      c->seq_len = keep + new_steps;
      c->allocated = true;
    }
    if ((rc = write(prev))) return rc;
    c->offset += S;
    return KVQ_OK;
  }

  const int64_t M = c->d.max_size;
  if (S == 1) {
    // #updateInPlace (:1026-1086)
    const int64_t prev = c->offset;
    if (!c->allocated || (prev >= c->seq_len && c->seq_len < M)) {
      const int64_t new_size = std::min<int64_t>(256, M - prev);
      if (new_size <= 0) return fail(KVQ_ERR_STATE, "rotating cache: offset beyond max_size with a short buffer");
      const int64_t keep = c->allocated ? c->seq_len : 0;
      if ((rc = grow_to(c, keep, keep + new_size, st))) return rc;
      c->seq_len = keep + new_size;
      c->allocated = true;
      c->ring_idx = prev;
    }
    const int64_t trim = c->seq_len - M;
    if (trim > 0) {
      // drop the oldest `trim` rows: buffer = buffer[trim:]
      if ((rc = relayout(c, round_up(std::max<int64_t>(M, c->d.reserve_rows), 16), {{trim, 0, M}}, st)))
        return rc;
      c->seq_len = M;
      c->ring_idx = M;
    }
    if (c->ring_idx == M) c->ring_idx = 0;
    if ((rc = write(c->ring_idx))) return rc;
    c->offset += 1;
    c->ring_idx += 1;
    return KVQ_OK;
  }

  // #updateConcat (:1003-1024): temporal order, trim to max_size - 1, append S
  if (!c->allocated) {
    const int64_t cap = round_up(std::max<int64_t>({(int64_t)S, M, c->d.reserve_rows}), 16);
    if (!c->base || cap > c->cap) {
      if ((rc = relayout(c, cap, {}, st))) return rc;
    } else if ((rc = zero_rows(c, 0, c->cap, st))) {
      return rc;
    }
    c->allocated = true;
    if ((rc = write(0))) return rc;
    c->seq_len = S;
  } else {
    std::vector<Seg> order;  // temporal order of the current buffer
    if (c->ring_idx == c->seq_len) {
      order.push_back({0, 0, c->seq_len});
    } else if (c->ring_idx < c->offset) {
      order.push_back({c->ring_idx, 0, c->seq_len - c->ring_idx});
      order.push_back({0, c->seq_len - c->ring_idx, c->ring_idx});
    } else {
      order.push_back({0, 0, c->ring_idx});
    }
    int64_t T = 0;
    for (const Seg& s : order) T += s.rows;
    const int64_t skip = std::max<int64_t>(0, T - M + 1);
    // drop the first `skip` temporal rows
    std::vector<Seg> segs;
    int64_t dropped = 0, dst = 0;
    for (const Seg& s : order) {
      int64_t src = s.src_row, rows = s.rows;
      const int64_t cut = std::min(rows, skip - dropped);
      if (cut > 0) {
        src += cut;
        rows -= cut;
        dropped += cut;
      }
      if (rows > 0) {
        segs.push_back({src, dst, rows});
        dst += rows;
      }
    }
    const int64_t new_len = dst + S;
    const int64_t cap = round_up(std::max<int64_t>({new_len, M, c->d.reserve_rows}), 16);
    if ((rc = relayout(c, cap, segs, st))) return rc;
    if ((rc = write(dst))) return rc;
    c->seq_len = new_len;
  }
  c->offset += S;
  c->ring_idx = c->seq_len;
  return KVQ_OK;
}

}  // namespace

extern "C" {

const char* kvq_last_error(void) { return g_last_error.c_str(); }

int32_t kvq_version(void) { return 100; }

int32_t kvq_cache_create(const kvq_desc* desc, kvq_cache** out) {
  if (!out) return fail(KVQ_ERR_ARG, "out is NULL");
  *out = nullptr;
  int32_t rc = check_desc(desc);
  if (rc) return rc;
  kvq_cache* c = new kvq_cache();
  c->d = *desc;
  if (desc->reserve_rows > 0) {
    DeviceGuard g(desc->device);
    if (!g.ok) {
      delete c;
      return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
    }
    int64_t cap = round_up(std::max<int64_t>(desc->reserve_rows, desc->max_size), c->ring() ? 16 : 256);
    rc = relayout(c, cap, {}, nullptr);
    if (rc) {
      delete c;
      return rc;
    }
  }
  *out = c;
  return KVQ_OK;
}

int32_t kvq_cache_free(kvq_cache* c) {
  if (!c) return KVQ_OK;
  int32_t rc = KVQ_OK;
  if (c->base) {
    DeviceGuard g(c->d.device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaFree(c->base);
    if (e != cudaSuccess) rc = cuda_fail(e, "cudaFree(cache)");
  }
  delete c;
  return rc;
}

int32_t kvq_append(kvq_cache* c, const void* k, const void* v, int32_t S, const int64_t* k_strides,
                   const int64_t* v_strides, void* stream) {
  if (!c) return fail(KVQ_ERR_ARG, "cache is NULL");
  if (!k || !v || !k_strides || !v_strides) return fail(KVQ_ERR_ARG, "NULL k / v / strides");
  if (S <= 0) return fail(KVQ_ERR_ARG, "S must be positive");
  if (k_strides[3] != 1 || v_strides[3] != 1) return fail(KVQ_ERR_ARG, "the d stride of k and v must be 1");
  DeviceGuard guard(c->d.device);
  if (!guard.ok) return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return append_rows(c, S, st, [&](int64_t dst) {
    return quantize_into(c, k, v, S, k_strides, v_strides, dst, st);
  });
}

}  // extern "C"

namespace {

int32_t check_qlinear(const kvq_qlinear& w, const char* name, const kvq_desc& d) {
  const std::string n(name);
  if (!w.packed || !w.scales) return fail(KVQ_ERR_ARG, n + ": NULL packed / scales");
  if (w.bits != 4 && w.bits != 8) return fail(KVQ_ERR_ARG, n + ": bits must be 4 or 8");
  if (w.group_size != 32 && w.group_size != 64 && w.group_size != 128)
    return fail(KVQ_ERR_ARG, n + ": group_size must be 32, 64 or 128");
  if (w.in_features <= 0 || w.in_features % w.group_size)
    return fail(KVQ_ERR_ARG, n + ": in_features must be a positive multiple of group_size");
  if ((int64_t)w.out_features != (int64_t)d.kv_heads * d.head_dim)
    return fail(KVQ_ERR_ARG, n + ": out_features must be its heads * head_dim");
  if (reinterpret_cast<uintptr_t>(w.packed) % 16)
    return fail(KVQ_ERR_ARG, n + ": packed must be 16-byte aligned");
  return KVQ_OK;
}

int32_t make_proj_args(const kvq_cache* c, const void* x, int32_t L, const kvq_kv_projection* pr,
                       kvq::ProjArgs& a) {
  if (!c) return fail(KVQ_ERR_ARG, "cache is NULL");
  if (!pr) return fail(KVQ_ERR_ARG, "projection is NULL");
  if (L <= 0) return fail(KVQ_ERR_ARG, "L must be positive");
  const kvq_desc& d = c->d;
  if (d.head_dim > 256) return fail(KVQ_ERR_ARG, "the fused projection supports head_dim <= 256");
  int32_t rc = check_qlinear(pr->k_proj, "k_proj", d);
  if (rc) return rc;
  if (!pr->v_from_k) {
    if ((rc = check_qlinear(pr->v_proj, "v_proj", d))) return rc;
    if (pr->v_proj.in_features != pr->k_proj.in_features)
      return fail(KVQ_ERR_ARG, "k_proj and v_proj must share in_features");
    if (pr->v_proj.bits != pr->k_proj.bits)
      return fail(KVQ_ERR_ARG, "k_proj and v_proj must share a bit width");
  }
  const bool has_q = pr->q_proj.packed != nullptr;
  if (has_q) {
    if (pr->q_heads <= 0) return fail(KVQ_ERR_ARG, "q_heads must be positive with a query projection");
    kvq_desc dq = d;
    dq.kv_heads = pr->q_heads;  // out_features = q_heads * head_dim
    if ((rc = check_qlinear(pr->q_proj, "q_proj", dq))) return rc;
    if (pr->q_proj.in_features != pr->k_proj.in_features)
      return fail(KVQ_ERR_ARG, "k_proj and q_proj must share in_features");
    if (pr->q_proj.bits != pr->k_proj.bits)
      return fail(KVQ_ERR_ARG, "k_proj and q_proj must share a bit width");
  }
  if (pr->rope_dims < 0 || pr->rope_dims > d.head_dim || pr->rope_dims % 2)
    return fail(KVQ_ERR_ARG, "rope_dims must be even and within head_dim");
  if (pr->rope_dims > 0 && !pr->rope_freqs && !(pr->rope_base > 0.0f))
    return fail(KVQ_ERR_ARG, "rope_base must be positive (or rope_freqs given)");
  a = kvq::ProjArgs{};
  a.x = x;
  a.B = d.batch;
  a.L = L;
  a.hidden = pr->k_proj.in_features;
  a.wk = {pr->k_proj.packed, pr->k_proj.scales, pr->k_proj.biases, pr->k_proj.bits, pr->k_proj.group_size};
  a.v_from_k = pr->v_from_k != 0;
  if (!a.v_from_k)
    a.wv = {pr->v_proj.packed, pr->v_proj.scales, pr->v_proj.biases, pr->v_proj.bits, pr->v_proj.group_size};
  a.has_q = has_q;
  if (has_q) {
    a.Hq = pr->q_heads;
    a.wq = {pr->q_proj.packed, pr->q_proj.scales, pr->q_proj.biases, pr->q_proj.bits,
            pr->q_proj.group_size};
  }
  a.k_norm = pr->k_norm_weight;
  a.v_norm = pr->v_norm_weight;
  a.q_norm = pr->q_norm_weight;
  a.norms = (pr->k_norm ? 1 : 0) | (pr->v_norm ? 2 : 0) | (has_q && pr->q_norm ? 4 : 0);
  a.eps = pr->norm_eps;
  a.rope_dims = pr->rope_dims;
  a.rope_traditional = pr->rope_traditional != 0;
  a.rope_base = pr->rope_base;
  a.rope_scale = pr->rope_scale;
  a.rope_pre_scale = pr->rope_pre_scale;
  a.rope_freqs = pr->rope_freqs;
  a.pos0 = c->offset;
  return KVQ_OK;
}

}  // namespace

extern "C" {

int32_t kvq_append_projected(kvq_cache* c, const void* x, int32_t L, const kvq_kv_projection* proj,
                             void* q_out, void* k_out, void* v_out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  kvq::ProjArgs a;
  int32_t rc = make_proj_args(c, x, L, proj, a);
  if (rc) return rc;
  if (!x) return fail(KVQ_ERR_ARG, "x is NULL");
  if (a.has_q && !q_out) return fail(KVQ_ERR_ARG, "q_out is NULL with a query projection");
  a.q_out = q_out;
  a.k_out = k_out;
  a.v_out = v_out;
  DeviceGuard guard(c->d.device);
  if (!guard.ok) return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (workspace) {
    const size_t need = kvq::project_workspace_bytes(a, c->d.kv_heads, c->d.head_dim, nullptr);
    if (workspace_bytes < need)
      return fail(KVQ_ERR_WORKSPACE, "workspace too small: " + std::to_string(need) + " bytes needed");
  }
  RowGeom g{c->d.head_dim, c->d.bits, c->d.group_size};
  return append_rows(c, L, st, [&](int64_t dst) {
    return kvq::launch_project_append(a, c->d.kv_heads, g, c->d.dtype, c->k, c->v, dst, workspace,
                                      workspace_bytes, st);
  });
}

int32_t kvq_append_projected_workspace(const kvq_cache* c, int32_t L, const kvq_kv_projection* proj,
                                       size_t* bytes) {
  if (!bytes) return fail(KVQ_ERR_ARG, "bytes is NULL");
  kvq::ProjArgs a;
  int32_t rc = make_proj_args(c, nullptr, L, proj, a);
  if (rc) return rc;
  DeviceGuard guard(c->d.device);
  if (!guard.ok) return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
  *bytes = kvq::project_workspace_bytes(a, c->d.kv_heads, c->d.head_dim, nullptr);
  return KVQ_OK;
}

int32_t kvq_cache_fetch(const kvq_cache* c, kvq_qtensor* keys, kvq_qtensor* values) {
  if (!c || !keys || !values) return fail(KVQ_ERR_ARG, "NULL argument");
  if (!c->allocated) return fail(KVQ_ERR_STATE, "cache is empty");
  int64_t len = c->offset;
  if (c->ring()) len = c->offset < c->d.max_size ? c->offset : c->seq_len;
  const TripleView* tv[2] = {&c->k, &c->v};
  kvq_qtensor* out[2] = {keys, values};
  for (int i = 0; i < 2; i++) {
    kvq_qtensor& t = *out[i];
    t.packed = tv[i]->packed;
    t.scales = tv[i]->scales;
    t.biases = tv[i]->biases;
    t.batch_stride = tv[i]->batch_stride;
    t.head_stride = tv[i]->head_stride;
    t.batch = c->d.batch;
    t.heads = c->d.kv_heads;
    t.len = (int32_t)len;
    t.head_dim = c->d.head_dim;
    t.bits = c->d.bits;
    t.group_size = c->d.group_size;
    t.dtype = c->d.dtype;
  }
  return KVQ_OK;
}

int32_t kvq_cache_state(const kvq_cache* c, int64_t* offset, int64_t* ring_idx, int64_t* seq_len,
                        int64_t* capacity) {
  if (!c) return fail(KVQ_ERR_ARG, "cache is NULL");
  if (offset) *offset = c->offset;
  if (ring_idx) *ring_idx = c->ring() ? c->ring_idx : c->offset;
  if (seq_len) *seq_len = c->allocated ? c->seq_len : 0;
  if (capacity) *capacity = c->base ? c->cap : 0;
  return KVQ_OK;
}

int32_t kvq_cache_trim(kvq_cache* c, int32_t n, int32_t bypass) {
  if (!c) return fail(KVQ_ERR_ARG, "cache is NULL");
  if (n < 0) return fail(KVQ_ERR_ARG, "n must be >= 0");
  if (!c->ring()) {
    c->offset = std::max<int64_t>(0, c->offset - n);
    return KVQ_OK;
  }
  const int64_t k = std::min<int64_t>(c->offset, n);
  if (!bypass) {
    c->offset -= k;
    c->ring_idx -= k;
    return KVQ_OK;
  }
  c->offset -= k;
  if (k > 0 && c->allocated) {
    c->seq_len -= k;
    c->ring_idx = c->seq_len;
  } else {
    c->ring_idx -= k;
  }
  return KVQ_OK;
}

int32_t kvq_cache_make_mask(const kvq_cache* c, int32_t N, int32_t window_size, int32_t* mask_mode,
                            int32_t* mask_window) {
  if (!c || !mask_mode || !mask_window) return fail(KVQ_ERR_ARG, "NULL argument");
  if (N <= 0) return fail(KVQ_ERR_ARG, "N must be positive");
  *mask_mode = KVQ_MASK_NONE;
  *mask_window = 0;
  if (N == 1) return KVQ_OK;
  if (!c->ring()) {
    *mask_mode = KVQ_MASK_CAUSAL;
    *mask_window = window_size > 0 ? window_size : 0;
    return KVQ_OK;
  }
  const int64_t w = window_size > 0 ? window_size : c->d.max_size;
  const int64_t off = std::min<int64_t>(c->d.max_size - 1, c->offset);
  *mask_mode = KVQ_MASK_CAUSAL;
  *mask_window = (off + N > w) ? (int32_t)w : 0;
  return KVQ_OK;
}

int32_t kvq_append_ragged(kvq_cache* c, const void* k, const void* v, int32_t S,
                          const int64_t* k_strides, const int64_t* v_strides, int32_t* seq_lens,
                          const int32_t* counts, void* stream) {
  if (!c) return fail(KVQ_ERR_ARG, "cache is NULL");
  if (!k || !v || !k_strides || !v_strides || !seq_lens)
    return fail(KVQ_ERR_ARG, "NULL k / v / strides / seq_lens");
  if (S <= 0) return fail(KVQ_ERR_ARG, "S must be positive");
  if (k_strides[3] != 1 || v_strides[3] != 1) return fail(KVQ_ERR_ARG, "the d stride of k and v must be 1");
  if (c->ring()) return fail(KVQ_ERR_STATE, "ragged appends take growing caches (max_size 0)");
  if (!c->base)
    return fail(KVQ_ERR_STATE, "ragged appends need the rows reserved at creation (reserve_rows > 0)");
  DeviceGuard guard(c->d.device);
  if (!guard.ok) return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
  RowGeom g{c->d.head_dim, c->d.bits, c->d.group_size};
  return launch_append_ragged(k, k_strides, v, v_strides, c->d.batch, c->d.kv_heads, S, g,
                              c->d.dtype, c->k, c->v, c->cap, seq_lens, counts, c->status,
                              static_cast<cudaStream_t>(stream));
}

int32_t kvq_cache_fetch_all(const kvq_cache* c, kvq_qtensor* keys, kvq_qtensor* values) {
  if (!c || !keys || !values) return fail(KVQ_ERR_ARG, "NULL argument");
  if (!c->base) return fail(KVQ_ERR_STATE, "cache has no device storage yet");
  const TripleView* tv[2] = {&c->k, &c->v};
  kvq_qtensor* out[2] = {keys, values};
  for (int i = 0; i < 2; i++) {
    kvq_qtensor& t = *out[i];
    t.packed = tv[i]->packed;
    t.scales = tv[i]->scales;
    t.biases = tv[i]->biases;
    t.batch_stride = tv[i]->batch_stride;
    t.head_stride = tv[i]->head_stride;
    t.batch = c->d.batch;
    t.heads = c->d.kv_heads;
    t.len = (int32_t)c->cap;
    t.head_dim = c->d.head_dim;
    t.bits = c->d.bits;
    t.group_size = c->d.group_size;
    t.dtype = c->d.dtype;
  }
  return KVQ_OK;
}

int32_t kvq_cache_check(kvq_cache* c, void* stream) {
  if (!c) return fail(KVQ_ERR_ARG, "cache is NULL");
  if (!c->base) return KVQ_OK;
  DeviceGuard guard(c->d.device);
  KVQ_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int flag = 0;
  KVQ_CUDA_TRY(cudaMemcpy(&flag, c->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (flag) {
    const int zero = 0;
    KVQ_CUDA_TRY(cudaMemcpy(c->status, &zero, sizeof(int), cudaMemcpyHostToDevice));
    return fail(KVQ_ERR_STATE, "a ragged append would have passed the cache's capacity (rows skipped)");
  }
  return KVQ_OK;
}

int32_t kvq_cache_from_dense(const kvq_desc* desc, const void* k, const void* v, int32_t rows,
                             const int64_t* k_strides, const int64_t* v_strides, int64_t offset,
                             int64_t ring_idx, void* stream, kvq_cache** out) {
  if (!out) return fail(KVQ_ERR_ARG, "out is NULL");
  *out = nullptr;
  if (!desc) return fail(KVQ_ERR_ARG, "desc is NULL");
  if (rows > 0 && (!k || !v || !k_strides || !v_strides))
    return fail(KVQ_ERR_ARG, "NULL k / v / strides");
  if (rows > 0 && (k_strides[3] != 1 || v_strides[3] != 1))
    return fail(KVQ_ERR_ARG, "the d stride of k and v must be 1");
  DeviceGuard guard(desc->device);
  if (!guard.ok) return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  kvq_cache* c = nullptr;
  int32_t rc = adopt_state(desc, rows, offset, ring_idx, st, &c);
  if (rc) return rc;
  if (rows > 0 && (rc = quantize_into(c, k, v, rows, k_strides, v_strides, 0, st))) {
    kvq_cache_free(c);
    return rc;
  }
  *out = c;
  return KVQ_OK;
}

int32_t kvq_cache_export(const kvq_cache* c, int64_t rows, void* const* host, void* stream) {
  if (!c || !host) return fail(KVQ_ERR_ARG, "NULL argument");
  if (rows < 0 || (rows > 0 && (!c->base || rows > c->cap)))
    return fail(KVQ_ERR_ARG, "rows must lie in [0, capacity]");
  for (int i = 0; i < 6; i++)
    if (rows > 0 && !host[i]) return fail(KVQ_ERR_ARG, "NULL host buffer");
  if (rows == 0) return KVQ_OK;
  DeviceGuard guard(c->d.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  size_t rb[6];
  row_bytes(c, rb);
  for (int i = 0; i < 6; i++)
    KVQ_CUDA_TRY(cudaMemcpy2DAsync(host[i], rows * rb[i], comp_ptr(c, i), c->cap * rb[i],
                                   rows * rb[i], (size_t)c->bh(), cudaMemcpyDeviceToHost, st));
  KVQ_CUDA_TRY(cudaStreamSynchronize(st));
  return KVQ_OK;
}

int32_t kvq_cache_import(const kvq_desc* desc, const void* const* host, int32_t rows,
                         int64_t offset, int64_t ring_idx, void* stream, kvq_cache** out) {
  if (!out) return fail(KVQ_ERR_ARG, "out is NULL");
  *out = nullptr;
  if (!desc) return fail(KVQ_ERR_ARG, "desc is NULL");
  if (rows > 0 && !host) return fail(KVQ_ERR_ARG, "NULL host buffers");
  for (int i = 0; rows > 0 && i < 6; i++)
    if (!host[i]) return fail(KVQ_ERR_ARG, "NULL host buffer");
  DeviceGuard guard(desc->device);
  if (!guard.ok) return fail(KVQ_ERR_CUDA, "cannot select the cache's device");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  kvq_cache* c = nullptr;
  int32_t rc = adopt_state(desc, rows, offset, ring_idx, st, &c);
  if (rc) return rc;
  if (rows > 0) {
    size_t rb[6];
    row_bytes(c, rb);
    for (int i = 0; i < 6; i++) {
      const cudaError_t e = cudaMemcpy2DAsync(comp_ptr(c, i), c->cap * rb[i], host[i],
                                              rows * rb[i], rows * rb[i], (size_t)c->bh(),
                                              cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) {
        kvq_cache_free(c);
        return cuda_fail(e, "cudaMemcpy2DAsync(import)");
      }
    }
    const cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      kvq_cache_free(c);
      return cuda_fail(e, "cudaStreamSynchronize(import)");
    }
  }
  *out = c;
  return KVQ_OK;
}

int32_t kvq_quantize(const void* x, int64_t rows, int32_t head_dim, int32_t group_size,
                     int32_t bits, int32_t dtype, void* packed, void* scales, void* biases,
                     void* stream) {
  if (rows < 0) return fail(KVQ_ERR_ARG, "rows must be >= 0");
  if (rows == 0) return KVQ_OK;
  if (!x || !packed || !scales || !biases) return fail(KVQ_ERR_ARG, "NULL pointer");
  kvq_desc d{1, 1, head_dim, bits, group_size, dtype, 0, 0, 0};
  int32_t rc = check_desc(&d);
  if (rc) return rc;
  RowGeom g{head_dim, bits, group_size};
  return launch_quantize_rows(x, rows, g, dtype, static_cast<uint32_t*>(packed),
                              static_cast<uint16_t*>(scales), static_cast<uint16_t*>(biases),
                              static_cast<cudaStream_t>(stream));
}

int32_t kvq_sdpa_decode_workspace(const kvq_qtensor* keys, int32_t q_heads, size_t* bytes) {
  if (!keys || !bytes) return fail(KVQ_ERR_ARG, "NULL argument");
  if (keys->heads <= 0 || q_heads <= 0 || q_heads % keys->heads)
    return fail(KVQ_ERR_ARG, "q_heads must be a positive multiple of kv heads");
  *bytes = decode_workspace_bytes(keys->batch, keys->heads, q_heads, keys->len, keys->head_dim);
  return KVQ_OK;
}

int32_t kvq_sdpa_decode(const kvq_qtensor* keys, const kvq_qtensor* values, const void* q,
                        int32_t q_heads, float scale, const int32_t* seq_lens, void* out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  AttnArgs a{};
  int32_t rc = make_attn_args(keys, values, q, q_heads, scale, seq_lens, a);
  if (rc) return rc;
  if (!out) return fail(KVQ_ERR_ARG, "out is NULL");
  return launch_decode(a, out, nullptr, nullptr, nullptr, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int32_t kvq_sdpa_decode_partial(const kvq_qtensor* keys, const kvq_qtensor* values,
                                const void* q, int32_t q_heads, float scale,
                                const int32_t* seq_lens, float* m, float* l, float* o,
                                void* workspace, size_t workspace_bytes, void* stream) {
  AttnArgs a{};
  int32_t rc = make_attn_args(keys, values, q, q_heads, scale, seq_lens, a);
  if (rc) return rc;
  if (!m || !l || !o) return fail(KVQ_ERR_ARG, "NULL partial output");
  return launch_decode(a, nullptr, m, l, o, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int32_t kvq_sdpa_merge(const float* m, const float* l, const float* o, int32_t parts,
                       int64_t part_stride, int32_t rows, int32_t head_dim, int32_t dtype,
                       void* out, void* stream) {
  if (!m || !l || !o || !out) return fail(KVQ_ERR_ARG, "NULL argument");
  if (parts <= 0 || rows < 0 || head_dim <= 0 || part_stride < 0) return fail(KVQ_ERR_ARG, "bad sizes");
  if (parts > 1 && part_stride < (int64_t)rows) return fail(KVQ_ERR_ARG, "part_stride smaller than rows");
  if (dtype != KVQ_DTYPE_FLOAT16 && dtype != KVQ_DTYPE_BFLOAT16) return fail(KVQ_ERR_ARG, "bad dtype");
  return launch_merge(m, l, o, parts, part_stride, rows, head_dim, dtype, out,
                      static_cast<cudaStream_t>(stream));
}

int32_t kvq_sdpa_prefill(const kvq_qtensor* keys, const kvq_qtensor* values, const void* q,
                         int32_t q_heads, int32_t L, float scale, int32_t mask_mode,
                         int32_t window, void* out, void* workspace, size_t workspace_bytes,
                         void* stream) {
  AttnArgs a{};
  int32_t rc = make_attn_args(keys, values, q, q_heads, scale, nullptr, a);
  if (rc) return rc;
  if (!out) return fail(KVQ_ERR_ARG, "out is NULL");
  if (mask_mode != KVQ_MASK_NONE && mask_mode != KVQ_MASK_CAUSAL) return fail(KVQ_ERR_ARG, "bad mask_mode");
  if (window < 0) return fail(KVQ_ERR_ARG, "window must be >= 0");
  return launch_prefill(a, L, mask_mode, mask_mode == KVQ_MASK_CAUSAL ? window : 0, out, workspace,
                        workspace_bytes, static_cast<cudaStream_t>(stream));
}

int32_t kvq_debug_scores(const kvq_qtensor* keys, const void* q, int32_t q_heads, int32_t L,
                         float scale, int32_t mask_mode, int32_t window, float* scores,
                         void* stream) {
  AttnArgs a{};
  int32_t rc = make_attn_args(keys, keys, q, q_heads, scale, nullptr, a);
  if (rc) return rc;
  if (!scores || L <= 0 || L > keys->len) return fail(KVQ_ERR_ARG, "bad scores / L");
  return launch_debug_scores(a, L, mask_mode, mask_mode == KVQ_MASK_CAUSAL ? window : 0, scores,
                             static_cast<cudaStream_t>(stream));
}

int32_t kvq_check_device(void* workspace, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KVQ_CUDA_TRY(cudaStreamSynchronize(st));
  std::vector<void*> flags;
  if (workspace) {
    flags.push_back(workspace);
  } else {
    int dev = 0;
    KVQ_CUDA_TRY(cudaGetDevice(&dev));
    flags = managed_ptrs(dev);
    if (void* s = noalloc_scratch_if_known(dev)) flags.push_back(s);
  }
  bool raised = false;
  for (void* f : flags) {
    int flag = 0;
    KVQ_CUDA_TRY(cudaMemcpy(&flag, f, sizeof(int), cudaMemcpyDeviceToHost));
    if (flag) {
      const int zero = 0;
      KVQ_CUDA_TRY(cudaMemcpy(f, &zero, sizeof(int), cudaMemcpyHostToDevice));
      raised = true;
    }
  }
  if (raised)
    return fail(KVQ_ERR_CUDA, "a kernel gave up waiting for its TMA copies (device error flag set)");
  return KVQ_OK;
}

int32_t kvq_debug_raise_flag(void* workspace, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<void*> flags;
  if (workspace) {
    flags.push_back(workspace);
  } else {
    int dev = 0;
    KVQ_CUDA_TRY(cudaGetDevice(&dev));
    flags = managed_ptrs(dev);
    if (void* s = noalloc_scratch_if_known(dev)) flags.push_back(s);
  }
  for (void* f : flags) KVQ_CUDA_TRY(cudaMemsetAsync(f, 1, 1, st));
  return KVQ_OK;
}

}  // extern "C"
