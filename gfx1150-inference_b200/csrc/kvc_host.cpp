// Host runtime of libkvcache.so: the C ABI declared in include/kvcache.h.
//
// Ownership and threading follow the reference's FFI layer
// (src/python_bindings/bindings.cpp): the native side owns device memory, every
// reference-compatible entry point runs under one process-wide mutex
// (bindings.cpp:18), and errors come back as status codes whose classes match
// the reference's exceptions (invalid_argument / out_of_range / runtime_error).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <mutex>
#include <queue>
#include <string>
#include <thread>
#include <vector>

#include "kvcache.h"
#include "kvc_common.h"
#include "kvc_internal.h"

using kvc::PoolGeom;

// ============================================================================
// errors
// ============================================================================
namespace kvc {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(KVC_ERR_CUDA, "CUDA error in %s - %s", what, cudaGetErrorString(e));
}

void clear_error() { g_last_error.clear(); }

// ---- bounded host waits ------------------------------------------------------
std::atomic<double> g_wait_limit_s{60.0};

namespace {
template <typename Query>
int bounded_wait(Query query, const char* what) {
  const double limit = g_wait_limit_s.load();
  if (injected_failure(KVC_FAULT_WAIT))
    return set_error(KVC_ERR_TIMEOUT, "%s did not complete within %.3f s (injected)", what, limit);
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned i = 0;; ++i) {
    const cudaError_t e = query();
    if (e == cudaSuccess) return KVC_OK;
    if (e != cudaErrorNotReady) return cuda_error(e, what);
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > limit)
      return set_error(KVC_ERR_TIMEOUT, "%s did not complete within %.3f s", what, limit);
    // spin first (most waits end within microseconds), then yield, then sleep
    if (i >= 4096) {
      std::this_thread::sleep_for(std::chrono::microseconds(dt > 0.01 ? 200 : 20));
    } else if (i >= 256) {
      std::this_thread::yield();
    }
  }
}
}  // namespace

int wait_stream(cudaStream_t s, const char* what) {
  return bounded_wait([s] { return cudaStreamQuery(s); }, what);
}

int wait_event(cudaEvent_t ev, const char* what) {
  return bounded_wait([ev] { return cudaEventQuery(ev); }, what);
}

// ---- host-side fault injection (kvc_test_inject_failure) ----------------------
namespace {
constexpr int kFaultSites = 5;
std::mutex g_fault_mu;
int g_fault_skip[kFaultSites] = {};
int g_fault_count[kFaultSites] = {};
std::atomic<int> g_fault_armed{0};
}  // namespace

bool injected_failure(int site) {
  if (g_fault_armed.load(std::memory_order_relaxed) == 0 || site <= 0 || site >= kFaultSites)
    return false;
  std::lock_guard<std::mutex> lock(g_fault_mu);
  if (g_fault_count[site] <= 0) return false;
  if (g_fault_skip[site] > 0) {
    g_fault_skip[site]--;
    return false;
  }
  if (--g_fault_count[site] == 0) g_fault_armed.fetch_sub(1);
  return true;
}

cudaError_t dev_alloc(void** p, size_t n) {
  if (injected_failure(KVC_FAULT_DEVICE_ALLOC)) return cudaErrorMemoryAllocation;
  return cudaMalloc(p, n);
}

cudaError_t host_alloc(void** p, size_t n, unsigned flags) {
  if (injected_failure(KVC_FAULT_HOST_ALLOC)) return cudaErrorMemoryAllocation;
  return cudaHostAlloc(p, n, flags);
}

cudaError_t host_register(void* p, size_t n) {
  if (injected_failure(KVC_FAULT_HOST_REGISTER)) return cudaErrorNotPermitted;
  return cudaHostRegister(p, n, cudaHostRegisterDefault);
}

std::atomic<uint32_t> g_device_errors{0};

int check_device_error(const char* what) {
  uint32_t code = 0, info = 0;
  cudaError_t e = read_device_error(&code, &info, true);
  if (e != cudaSuccess) return cuda_error(e, what);
  if (code == KVC_DEVERR_NONE) return KVC_OK;
  g_device_errors.fetch_add(1);
  const char* name = code == KVC_DEVERR_BAD_PAGE       ? "block table entry out of range"
                     : code == KVC_DEVERR_WAIT_LIMIT   ? "pipeline wait gave up after its time limit"
                     : code == KVC_DEVERR_BAD_POSITION ? "append position outside the block table"
                                                       : "unknown device error";
  return set_error(KVC_ERR_DEVICE, "%s: %s (value %d)", what, name, static_cast<int>(info));
}

void* mapped_host_ptr(void* h) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, h) != cudaSuccess) {
    cudaGetLastError();  // pageable memory on older runtimes reports an error
    return nullptr;
  }
  return attr.type == cudaMemoryTypeHost ? attr.devicePointer : nullptr;
}

namespace {
// Page-locked landing place of each device's error word, and the word's address.
struct ErrMirror {
  uint32_t* host = nullptr;      // page-locked copy of the device error word
  uint32_t* host_dev = nullptr;  // its device address (null: not mapped)
  void* dev = nullptr;           // the device error word
};
// The error-word copy the kernels of this thread's host-buffer call in progress
// store (DecodeArgs::err_host), between stage_host_call and finish_host_call.
thread_local uint32_t* t_err_host = nullptr;
std::mutex g_mirror_mu;
ErrMirror g_mirror[64];

cudaError_t error_mirror(ErrMirror** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mirror_mu);
  ErrMirror& m = g_mirror[dev];
  if (!m.host) {
    void* h = nullptr;
    if ((e = host_alloc(&h, 64, cudaHostAllocDefault)) != cudaSuccess) return e;
    memset(h, 0, 64);
    if ((e = device_error_address(&m.dev)) != cudaSuccess) {
      cudaFreeHost(h);
      return e;
    }
    m.host = static_cast<uint32_t*>(h);
    m.host_dev = static_cast<uint32_t*>(mapped_host_ptr(h));
  }
  *out = &m;
  return cudaSuccess;
}
}  // namespace

int prepare_host_call() {
  ErrMirror* m = nullptr;
  const cudaError_t e = error_mirror(&m);
  if (e != cudaSuccess) return cuda_error(e, "device error mirror");
  t_err_host = m->host_dev;
  return KVC_OK;
}

uint32_t* host_call_error_copy() { return t_err_host; }

int finish_host_call(cudaStream_t s, void* h_out, const void* d_out, size_t bytes,
                     const char* what, bool merged) {
  cudaError_t e;
  if (d_out && bytes && (e = cudaMemcpyAsync(h_out, d_out, bytes, cudaMemcpyDeviceToHost, s)))
    return cuda_error(e, "cudaMemcpyAsync(D2H)");
  ErrMirror* m = nullptr;
  if ((e = error_mirror(&m)) != cudaSuccess) return cuda_error(e, "device error mirror");
  // Concurrent calls on one device copy the same word into the same place: a call
  // sees at least every error raised before its own kernels finished.  When the
  // call's last kernel is a split merge, that merge stored the word there already
  // (no copy-engine round trip on the call's critical path).
  const bool stored = merged && t_err_host != nullptr && t_err_host == m->host_dev;
  t_err_host = nullptr;
  if (!stored &&
      (e = cudaMemcpyAsync(m->host, m->dev, 2 * sizeof(uint32_t), cudaMemcpyDeviceToHost, s)))
    return cuda_error(e, "cudaMemcpyAsync(error word)");
  if (const int rc = wait_stream(s, what)) return rc;
  if ((reinterpret_cast<volatile uint32_t*>(m->host)[0]) == KVC_DEVERR_NONE) return KVC_OK;
  const int rc = check_device_error(what);  // rare: read, clear and report
  reinterpret_cast<volatile uint32_t*>(m->host)[0] = KVC_DEVERR_NONE;  // the word is clear now
  return rc;
}

int stage_host_call(HostBuf& pinned, const void* const h_in[3], const size_t in_bytes[3],
                    uint8_t* const d_in[3], void* h_out, size_t out_bytes, cudaStream_t s,
                    HostCallStage* st) {
  // the error word's page-locked mirror exists before this call's kernels run
  if (const int rc = prepare_host_call()) return rc;
  auto al16 = [](size_t b) { return (b + 15) & ~static_cast<size_t>(15); };
  const void* src[3] = {nullptr, nullptr, nullptr};
  size_t need = 0;
  for (int i = 0; i < 3; ++i) {
    if (!in_bytes[i]) continue;
    src[i] = mapped_host_ptr(const_cast<void*>(h_in[i]));
    if (!src[i] || (reinterpret_cast<uintptr_t>(src[i]) & 15u)) {
      src[i] = nullptr;
      need += al16(in_bytes[i]);
    }
  }
  void* out_direct = out_bytes ? mapped_host_ptr(h_out) : nullptr;
  const size_t out_off = al16(need);
  const size_t total = out_off + (out_direct ? 0 : al16(out_bytes));
  uint8_t* hp = nullptr;
  uint8_t* dp = nullptr;
  if (total) {
    cudaError_t e = pinned.ensure(total);
    if (e != cudaSuccess) return cuda_error(e, "cudaMallocHost(call staging)");
    hp = static_cast<uint8_t*>(pinned.ptr);
    dp = static_cast<uint8_t*>(mapped_host_ptr(pinned.ptr));
    if (!dp) return set_error(KVC_ERR_CUDA, "page-locked staging is not mapped on the device");
  }
  size_t off = 0;
  for (int i = 0; i < 3; ++i) {
    if (!in_bytes[i] || src[i]) continue;
    memcpy(hp + off, h_in[i], in_bytes[i]);
    src[i] = dp + off;
    off += al16(in_bytes[i]);
  }
  StageArgs a;
  for (int i = 0; i < 3; ++i) {
    a.src[i] = static_cast<const uint8_t*>(src[i]);
    a.dst[i] = d_in[i];
    a.bytes[i] = src[i] ? in_bytes[i] : 0;
  }
  cudaError_t e = launch_stage_inputs(a, s);
  if (e != cudaSuccess) return cuda_error(e, "input staging kernel");
  st->out_dev = out_direct ? out_direct : (out_bytes ? dp + out_off : nullptr);
  st->out_bounce = out_direct ? nullptr : (out_bytes ? hp + out_off : nullptr);
  return KVC_OK;
}

int finish_staged_call(cudaStream_t s, void* h_out, const HostCallStage& st, size_t out_bytes,
                       const char* what, bool merged) {
  const int rc = finish_host_call(s, h_out, nullptr, 0, what, merged);
  if (rc) return rc;
  if (st.out_bounce && out_bytes) memcpy(h_out, st.out_bounce, out_bytes);
  return KVC_OK;
}

int use_device(int device) {
  const cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? KVC_OK : cuda_error(e, "cudaSetDevice");
}

int elem_size_of(int dtype) {
  switch (dtype) {
    case KVC_DTYPE_F16: return 2;
    case KVC_DTYPE_BF16: return 2;
    case KVC_DTYPE_F32: return 4;
    default: return 0;
  }
}

// Growth of a buffer that already exists gets 25 % headroom (64 KiB granules):
// plans grow a little every time a context crosses a split boundary, and a
// reallocation (cudaFree synchronises the device) per crossing would cost far
// more than the headroom.  First allocations are exact.
static size_t grown_size(size_t cap, size_t bytes) {
  if (cap == 0) return bytes;
  const size_t want = bytes + bytes / 4;
  return (want + 65535) & ~static_cast<size_t>(65535);
}

cudaError_t DevBuf::ensure(size_t bytes) {
  if (bytes <= cap) return cudaSuccess;
  const size_t n = grown_size(cap, bytes);
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  cap = 0;
  cudaError_t e = dev_alloc(&ptr, n);
  if (e != cudaSuccess) {
    ptr = nullptr;
    return e;
  }
  cap = n;
  return cudaSuccess;
}

void DevBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  cap = 0;
}

cudaError_t HostBuf::ensure(size_t bytes) {
  if (bytes <= cap) return cudaSuccess;
  const size_t n = grown_size(cap, bytes);
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  cap = 0;
  cudaError_t e = host_alloc(&ptr, n, cudaHostAllocDefault);
  if (e != cudaSuccess) {
    ptr = nullptr;
    return e;
  }
  cap = n;
  return cudaSuccess;
}

void HostBuf::release() {
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  cap = 0;
}

int make_geom(int num_layers, int num_pages, int page_size, int num_kv_heads, int head_dim,
              int dtype, PoolGeom* g) {
  if (num_layers <= 0 || num_pages <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return set_error(KVC_ERR_INVALID_ARG, "KV cache dimensions must all be positive.");
  const int es = elem_size_of(dtype);
  if (es == 0) return set_error(KVC_ERR_INVALID_ARG, "unsupported KV storage dtype %d.", dtype);
  if (page_size <= 0 || page_size % kSlab != 0)
    return set_error(KVC_ERR_INVALID_ARG, "page_size must be a positive multiple of 16 (got %d).",
                     page_size);
  if (head_dim > 256)
    return set_error(KVC_ERR_INVALID_ARG, "head_dim must be in (0, 256] (got %d).", head_dim);
  if ((head_dim * es) % 16 != 0)
    return set_error(KVC_ERR_INVALID_ARG,
                     "head_dim * element size must be a multiple of 16 bytes (got head_dim %d).",
                     head_dim);
  g->num_layers = num_layers;
  g->num_pages = num_pages;
  g->page_size = page_size;
  g->num_kv_heads = num_kv_heads;
  g->head_dim = head_dim;
  g->dtype = dtype;
  g->elem_size = es;
  g->layout = (es == 2) ? kLayoutCore : kLayoutLinear;
  g->page_head_bytes = static_cast<size_t>(page_size) * head_dim * es;
  g->page_bytes = g->page_head_bytes * num_kv_heads;
  g->layer_bytes = g->page_bytes * num_pages;
  return KVC_OK;
}

}  // namespace kvc

using namespace kvc;

// ============================================================================
// pool
// ============================================================================
namespace kvc {

int pool_alloc(kvc_pool* p, const PoolGeom& g, int device) {
  const size_t bytes = g.layer_bytes * g.num_layers;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  if (bytes > p->cap_bytes) {
    if (p->k) cudaFree(p->k);
    if (p->v) cudaFree(p->v);
    p->k = p->v = nullptr;
    p->cap_bytes = 0;
    e = dev_alloc(reinterpret_cast<void**>(&p->k), bytes);
    if (e != cudaSuccess) {
      p->k = nullptr;
      return cuda_error(e, "cudaMalloc(K pool)");
    }
    e = dev_alloc(reinterpret_cast<void**>(&p->v), bytes);
    if (e != cudaSuccess) {
      cudaFree(p->k);
      p->k = p->v = nullptr;
      return cuda_error(e, "cudaMalloc(V pool)");
    }
    p->cap_bytes = bytes;
  }
  p->g = g;
  p->device = device;
  return KVC_OK;
}

void pool_release(kvc_pool* p) {
  if (p->k) cudaFree(p->k);
  if (p->v) cudaFree(p->v);
  p->k = p->v = nullptr;
  p->cap_bytes = 0;
  p->io.release();
  p->io_host.release();
  p->g = PoolGeom();
}

}  // namespace kvc

extern "C" int kvc_version(void) { return 1; }

extern "C" int kvc_set_host_wait_limit(double seconds) {
  if (!(seconds > 0.0) || seconds > 86400.0)
    return set_error(KVC_ERR_INVALID_ARG, "the host wait limit must be in (0, 86400] seconds.");
  kvc::g_wait_limit_s.store(seconds);
  return KVC_OK;
}

extern "C" int kvc_test_inject_failure(int site, int skip, int count) {
  if (site <= 0 || site >= kvc::kFaultSites || skip < 0 || count < 0)
    return set_error(KVC_ERR_INVALID_ARG, "unknown fault site %d or negative counts.", site);
  std::lock_guard<std::mutex> lock(kvc::g_fault_mu);
  const bool was = kvc::g_fault_count[site] > 0, now = count > 0;
  kvc::g_fault_skip[site] = skip;
  kvc::g_fault_count[site] = count;
  if (now && !was) kvc::g_fault_armed.fetch_add(1);
  if (!now && was) kvc::g_fault_armed.fetch_sub(1);
  return KVC_OK;
}

extern "C" const char* kvc_last_error(void) { return g_last_error.c_str(); }

extern "C" int kvc_device_error(int device, int clear, uint32_t* code, uint32_t* info) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  e = read_device_error(code, info, clear != 0);
  if (e != cudaSuccess) return cuda_error(e, "read_device_error");
  if (code && *code != KVC_DEVERR_NONE) g_device_errors.fetch_add(1);
  return KVC_OK;
}

extern "C" int kvc_device_sm_count(int device, int* out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  cudaError_t e = cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cuda_error(e, "cudaDeviceGetAttribute");
  return KVC_OK;
}

extern "C" int kvc_pool_create(int num_layers, int num_pages, int page_size, int num_kv_heads,
                               int head_dim, int dtype, int device, kvc_pool_t** out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  *out = nullptr;
  PoolGeom g;
  int rc = make_geom(num_layers, num_pages, page_size, num_kv_heads, head_dim, dtype, &g);
  if (rc) return rc;
  kvc_pool* p = new kvc_pool();
  rc = pool_alloc(p, g, device);
  if (rc) {
    delete p;
    return rc;
  }
  *out = p;
  return KVC_OK;
}

extern "C" int kvc_pool_destroy(kvc_pool_t* pool) {
  if (!pool) return KVC_OK;
  cudaSetDevice(pool->device);
  pool_release(pool);
  delete pool;
  return KVC_OK;
}

extern "C" int kvc_pool_info(const kvc_pool_t* pool, void** k_base, void** v_base,
                             size_t* bytes_per_layer, size_t* bytes_per_page_head) {
  if (!pool) return set_error(KVC_ERR_INVALID_ARG, "pool must not be null.");
  if (k_base) *k_base = pool->k;
  if (v_base) *v_base = pool->v;
  if (bytes_per_layer) *bytes_per_layer = pool->g.layer_bytes;
  if (bytes_per_page_head) *bytes_per_page_head = pool->g.page_head_bytes;
  return KVC_OK;
}

extern "C" int kvc_pool_fill_normal(kvc_pool_t* pool, int layer_begin, int layer_end,
                                    int page_begin, int page_end, uint64_t seed, float stddev,
                                    void* stream) {
  if (!pool) return set_error(KVC_ERR_INVALID_ARG, "pool must not be null.");
  const PoolGeom& g = pool->g;
  if (layer_begin < 0 || layer_end > g.num_layers || layer_begin > layer_end || page_begin < 0 ||
      page_end > g.num_pages || page_begin > page_end)
    return set_error(KVC_ERR_OUT_OF_RANGE, "fill range outside the pool.");
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t elems_per_page = g.page_bytes / g.elem_size;
  const size_t elems_per_layer = g.layer_bytes / g.elem_size;
  for (int l = layer_begin; l < layer_end; ++l) {
    for (int kv = 0; kv < 2; ++kv) {
      FillArgs f;
      uint8_t* base = kv == 0 ? pool->k : pool->v;
      f.base = base + static_cast<size_t>(l) * g.layer_bytes +
               static_cast<size_t>(page_begin) * g.page_bytes;
      f.n_elems = elems_per_page * static_cast<size_t>(page_end - page_begin);
      f.seed = seed + static_cast<uint64_t>(kv) * 0x5851F42D4C957F2Dull;
      f.index0 = static_cast<uint64_t>(l) * elems_per_layer +
                 static_cast<uint64_t>(page_begin) * elems_per_page;
      f.stddev = stddev;
      f.dtype = g.dtype;
      cudaError_t e = launch_fill_normal(f, s);
      if (e != cudaSuccess) return cuda_error(e, "fill_normal_kernel");
    }
  }
  return KVC_OK;
}

namespace kvc {

int do_append(kvc_pool* pool, int layer, const void* d_k_new, const void* d_v_new,
              const int32_t* d_bt, int bt_stride, const int32_t* d_rows, const int32_t* d_pos,
              int pos0, int n, cudaStream_t s) {
  const PoolGeom& g = pool->g;
  if (layer < 0 || layer >= g.num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for the KV pool.");
  if (n < 0) return set_error(KVC_ERR_INVALID_ARG, "row count must be non-negative.");
  if (n == 0) return KVC_OK;
  if (!d_k_new || !d_v_new || !d_bt)
    return set_error(KVC_ERR_INVALID_ARG, "K/V rows and block tables must not be null.");
  if ((reinterpret_cast<uintptr_t>(d_k_new) | reinterpret_cast<uintptr_t>(d_v_new)) & 15u)
    return set_error(KVC_ERR_INVALID_ARG, "K/V row buffers must be 16-byte aligned.");
  if (bt_stride <= 0) return set_error(KVC_ERR_INVALID_ARG, "bt_stride must be positive.");
  AppendArgs a;
  a.k_layer = pool->k + static_cast<size_t>(layer) * g.layer_bytes;
  a.v_layer = pool->v + static_cast<size_t>(layer) * g.layer_bytes;
  a.k_new = static_cast<const uint8_t*>(d_k_new);
  a.v_new = static_cast<const uint8_t*>(d_v_new);
  a.block_tables = d_bt;
  a.rows = d_rows;
  a.positions = d_pos;
  a.pos0 = pos0;
  a.bt_stride = bt_stride;
  a.n = n;
  a.num_kv_heads = g.num_kv_heads;
  a.row_units = g.head_dim * g.elem_size / 16;
  a.page_size = g.page_size;
  a.num_pages = g.num_pages;
  a.layout = g.layout;
  a.page_head_bytes = g.page_head_bytes;
  cudaError_t e = launch_append(a, g.elem_size, s);
  if (e != cudaSuccess) return cuda_error(e, "append_kernel");
  return KVC_OK;
}

}  // namespace kvc

extern "C" int kvc_append(kvc_pool_t* pool, int layer, const void* d_k_new, const void* d_v_new,
                          const int32_t* d_block_tables, int bt_stride, const int32_t* d_rows,
                          const int32_t* d_positions, int n, void* stream) {
  if (!pool) return set_error(KVC_ERR_INVALID_ARG, "pool must not be null.");
  if (!d_positions) return set_error(KVC_ERR_INVALID_ARG, "positions must not be null.");
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  return do_append(pool, layer, d_k_new, d_v_new, d_block_tables, bt_stride, d_rows, d_positions,
                   0, n, static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_gather(kvc_pool_t* pool, int layer, const int32_t* d_block_tables,
                          int bt_stride, int row, int start, int count, void* d_k_out,
                          void* d_v_out, void* stream) {
  if (!pool) return set_error(KVC_ERR_INVALID_ARG, "pool must not be null.");
  const PoolGeom& g = pool->g;
  if (layer < 0 || layer >= g.num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for the KV pool.");
  if (start < 0 || count < 0 ||
      static_cast<int64_t>(start) + count > static_cast<int64_t>(bt_stride) * g.page_size)
    return set_error(KVC_ERR_OUT_OF_RANGE, "gather range outside the block table.");
  if (row < 0) return set_error(KVC_ERR_OUT_OF_RANGE, "row must be non-negative.");
  if ((reinterpret_cast<uintptr_t>(d_k_out) | reinterpret_cast<uintptr_t>(d_v_out)) & 15u)
    return set_error(KVC_ERR_INVALID_ARG, "output buffers must be 16-byte aligned.");
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  GatherArgs a;
  a.k_layer = pool->k + static_cast<size_t>(layer) * g.layer_bytes;
  a.v_layer = pool->v + static_cast<size_t>(layer) * g.layer_bytes;
  a.k_out = static_cast<uint8_t*>(d_k_out);
  a.v_out = static_cast<uint8_t*>(d_v_out);
  a.bt_row = d_block_tables + static_cast<size_t>(row) * bt_stride;
  a.bt_stride = bt_stride;
  a.start = start;
  a.count = count;
  a.num_kv_heads = g.num_kv_heads;
  a.row_units = g.head_dim * g.elem_size / 16;
  a.page_size = g.page_size;
  a.num_pages = g.num_pages;
  a.layout = g.layout;
  a.page_head_bytes = g.page_head_bytes;
  cudaError_t e = launch_gather(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "gather_kernel");
  return KVC_OK;
}

// ============================================================================
// plans
// ============================================================================
namespace kvc {

// Positions per split (a multiple of the page size, at most kMaxSplitPages
// pages).  The persistent grid has W = SMs x 8 warps; each (split, KV head,
// q-head chunk) unit runs on one warp, units longest first, handed out
// dynamically.  For each candidate length s the host estimates the decode time
// in position units:
//   max( sum_u (len_u + c0) / W ,  max_u len_u + c0 )  +  (units > W ? s / 4 : 0)
// (c0 = a unit's fixed cost: first-slab latency, q load, partial write; s / 4 =
// the expected idle tail of the last wave) over the default 512 and every
// length of at least kMinSplit positions whose units fit one wave, and picks the
// cheapest, the longest on ties.  Long, even contexts with few units get one wave of equal units
// (e.g. 8 x 32K positions on one KV head: 224-position splits, 1176 units on
// 1184 warps); large ragged batches get 512-position splits and rely on the
// dynamic schedule.  The choice depends only on the context lengths and head
// counts of the batch, so the same call always gets the same partition (the
// resident and offloaded paths agree bit for bit).  KVC_SPLIT_TOKENS overrides
// it for tuning.
int l2_ahead_slabs(int split_tokens, bool even_ctx) {
  static int forced = [] {
    const char* e = getenv("KVC_L2_AHEAD");
    if (!e) return -1;
    const int x = atoi(e);
    return x < 0 ? 0 : (x > 32 ? 32 : x);
  }();
  if (forced >= 0) return forced;
  return (even_ctx && split_tokens >= kL2AheadMinSplit) ? kL2AheadSlabs : 0;
}

int split_tokens_for(int page_size) {
  static int base = [] {
    const char* e = getenv("KVC_SPLIT_TOKENS");
    int v = e ? atoi(e) : 0;
    if (v < 0) v = 0;
    if (v > 0 && v < kSlab) v = kSlab;
    return v;
  }();
  return base;  // 0: automatic
}

int round_split(int c, int page_size) {
  c = ((c + page_size - 1) / page_size) * page_size;
  while (c / page_size > kMaxSplitPages) c -= page_size;
  if (c > kMaxSplitPages * kSlab) c = (kMaxSplitPages * kSlab / page_size) * page_size;
  return c < page_size ? page_size : c;
}

int split_tokens_model(int page_size, const int* ctx, int n_queries, int units_per_split,
                       int sms) {
  const double warps = static_cast<double>(sms) * kPersistWarpsPerSm;
  constexpr double kUnitCost = 64.0;   // c0, in positions
  // Units of fewer than 8 slabs cost more than the model says: config 2 (one
  // 4,096-position MHA sequence) ran 1.3 % faster per step with 128-position
  // splits (1,024 units) than with the 112 (1,184 units) the model picks from 64 up,
  // and 7 % faster over its growing contexts 4,097-4,196 (A/B on one B200).
  constexpr int kMinSplit = 128;
  int64_t total = 0, max_ctx = 1;
  for (int i = 0; i < n_queries; ++i) {
    total += std::max(ctx[i], 1);
    max_ctx = std::max<int64_t>(max_ctx, ctx[i]);
  }
  const int s_lo = round_split(kMinSplit, page_size);
  const int s_hi = round_split(kMaxSplitPages * page_size, page_size);
  int best = round_split(kSplitTokens, page_size);
  double best_cost = -1.0;
  for (int sp = s_hi; sp >= s_lo; sp -= page_size) {
    int64_t units = 0;
    for (int i = 0; i < n_queries; ++i) units += ctx[i] > 0 ? (ctx[i] + sp - 1) / sp : 1;
    units *= units_per_split;
    const double work = (static_cast<double>(total) * units_per_split + kUnitCost * units) / warps;
    const double longest = static_cast<double>(std::min<int64_t>(sp, max_ctx)) + kUnitCost;
    // multi-wave partitions other than the default one are not considered
    if (units > warps && sp != round_split(kSplitTokens, page_size)) continue;
    const double cost = std::max(work, longest) + (units > warps ? 0.25 * sp : 0.0);
    if (best_cost < 0.0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

int device_sms(int device) {
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();  // the query's error must not surface as a later launch failure
    sms = 148;
  }
  return sms;
}

int choose_split_tokens(int page_size, const int* ctx, int n_queries, int units_per_split,
                        int sms) {
  const int forced = split_tokens_for(page_size);
  if (forced > 0) return round_split(forced, page_size);
  return split_tokens_model(page_size, ctx, n_queries, units_per_split, sms);
}

// Tail refinement: with even contexts (nothing but full splits), a multi-wave
// plan whose last wave would keep fewer than 60 % of the warps busy has that
// many full splits (the queries' last ones, round-robin) cut into quarters, so
// the end of the longest-first list is short units that every warp can take.
// Measured on config 4 (4,096 full units on 1,184 warps): +7 %; ragged batches
// already end in short splits and only pay the extra units (config 3: -4 % to
// -9 %), so they are left alone.  KVC_TAIL_REFINE = n overrides the count.
int split_partition(int page_size, const int* ctxs, int n_queries, int ups, int device,
                    int* refine) {
  return split_partition_sms(page_size, ctxs, n_queries, ups, device_sms(device), refine);
}

int split_partition_sms(int page_size, const int* ctxs, int n_queries, int ups, int sms,
                        int* refine) {
  const int C = choose_split_tokens(page_size, ctxs, n_queries, ups, sms);
  for (int i = 0; i < n_queries; ++i) refine[i] = 0;
  static const int forced = [] {
    const char* e = getenv("KVC_TAIL_REFINE");
    return e ? std::max(0, atoi(e)) : -1;
  }();
  int n_refine = forced;
  if (n_refine < 0) {
    n_refine = 0;
    const int64_t warps = static_cast<int64_t>(sms) * kPersistWarpsPerSm;
    int64_t full_units = 0, partial_pos = 0;
    for (int i = 0; i < n_queries; ++i) {
      full_units += static_cast<int64_t>(std::max(0, ctxs[i]) / C) * ups;
      partial_pos += static_cast<int64_t>(std::max(0, ctxs[i]) % C) * ups;
    }
    const int64_t r = full_units % warps;
    if (full_units > warps && r > 0 && r < (warps * 6) / 10 &&
        partial_pos * 20 < static_cast<int64_t>(C) * warps)
      n_refine = static_cast<int>((r + ups - 1) / ups);
  }
  const int q4 = C / 4;
  if (n_refine > 0 && q4 >= page_size && q4 % page_size == 0) {
    int left = n_refine;
    for (int round = 0; left > 0; ++round) {
      bool any = false;
      for (int i = 0; i < n_queries && left > 0; ++i) {
        const int full = std::max(0, ctxs[i]) / C;
        if (round < full) {
          refine[i]++;
          left--;
          any = true;
        }
      }
      if (!any) break;
    }
  }
  return C;
}

// Build the split list on the host.  ctx_of(i) / row_of(i) describe query i.
template <typename CtxFn, typename RowFn>
int plan_build(kvc_plan* p, const PoolGeom& g, int n_queries, int num_heads, CtxFn ctx_of,
               RowFn row_of, int device, cudaStream_t s) {
  if (n_queries < 0) return set_error(KVC_ERR_INVALID_ARG, "n_queries must be non-negative.");
  if (num_heads <= 0 || num_heads % g.num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be divisible by num_kv_heads.");
  if ((p->flags & KVC_PLAN_GRAPH) &&
      (!decode_uses_mma(g.dtype, g.head_dim, g.page_size) || g.layout != kLayoutCore))
    return set_error(KVC_ERR_INVALID_ARG,
                     "KVC_PLAN_GRAPH needs fp16/bf16 KV with head_dim in {32,64,96,128,160,192,256} "
                     "and a page size multiple of 16.");
  std::vector<int> ctxs(std::max(0, n_queries));
  for (int i = 0; i < n_queries; ++i) ctxs[i] = ctx_of(i);
  std::vector<int32_t> inputs = {n_queries, num_heads, g.num_kv_heads, g.head_dim, g.page_size,
                                 g.dtype, device};
  inputs.reserve(inputs.size() + 2 * static_cast<size_t>(std::max(0, n_queries)));
  for (int i = 0; i < n_queries; ++i) inputs.push_back(ctxs[i]);
  for (int i = 0; i < n_queries; ++i) inputs.push_back(row_of(i));
  // a kernel that gave up may have left the plan's unit counter armed: rebuild
  inputs.push_back(static_cast<int32_t>(g_device_errors.load()));
  if (p->valid && inputs == p->built_from) {
    p->pool_geom = g;
    return KVC_OK;
  }
  p->valid = false;
  p->built_from.clear();
  const int ups = g.num_kv_heads * ((num_heads / g.num_kv_heads + 7) / 8);
  std::vector<int> refine(std::max(0, n_queries), 0);  // full splits to quarter, per query
  const int C = split_partition(g.page_size, ctxs.data(), n_queries, ups, device, refine.data());
  p->items.clear();
  p->qinfo.clear();
  p->rows.clear();
  p->positions.clear();
  int slot = 0, max_ctx = 0, min_ctx = n_queries > 0 ? ctxs[0] : 0, max_splits = 0;
  for (int i = 0; i < n_queries; ++i) {
    const int ctx = ctxs[i];
    const int row = row_of(i);
    if (ctx < 0) return set_error(KVC_ERR_INVALID_ARG, "context length must be non-negative.");
    if (row < 0) return set_error(KVC_ERR_INVALID_ARG, "block-table row must be non-negative.");
    const int ns = emit_splits(i, ctx, C, refine[i], [&](const int4& it) { p->items.push_back(it); });
    p->qinfo.push_back(make_int4(row, ctx, slot, ns));
    p->rows.push_back(row);
    p->positions.push_back(ctx - 1);
    slot += ns;
    max_ctx = std::max(max_ctx, ctx);
    min_ctx = std::min(min_ctx, ctx);
    max_splits = std::max(max_splits, ns);
  }
  // Longest splits first: CTAs are dispatched roughly in index order, so the
  // short tail splits fill the last wave.
  std::stable_sort(p->items.begin(), p->items.end(), [](const int4& x, const int4& y) {
    return (x.w - x.z) > (y.w - y.z);
  });
  // Each kernel work item is {split record, its query's record}: one 32-byte load.
  p->item_pairs.resize(2 * p->items.size());
  for (size_t k = 0; k < p->items.size(); ++k) {
    p->item_pairs[2 * k] = p->items[k];
    p->item_pairs[2 * k + 1] = p->qinfo[p->items[k].x];
  }
  // Persistent schedule: units (item x KV head x q-head chunk) stored longest
  // first (items are sorted by length); the kernel hands them out dynamically.
  // Each unit is a self-contained 3 x int4 record.
  {
    const int sms = device_sms(device);
    const int group = num_heads / g.num_kv_heads;
    const int nhc = (group + 7) / 8;
    const int per_item = g.num_kv_heads * nhc;
    const int n_units = static_cast<int>(p->items.size()) * per_item;
    const int n_ctas = std::max(1, std::min(sms * kPersistCtasPerSm,
                                            (n_units + kPersistWarps - 1) / kPersistWarps));
    p->sched_recs.clear();
    for (int k = 0; k < static_cast<int>(p->items.size()); ++k) {
      const int4 it = p->items[k];
      for (int r = 0; r < per_item; ++r) {
        const int kvh = r / nhc, hc = r % nhc;
        p->sched_recs.push_back(it);
        p->sched_recs.push_back(p->qinfo[it.x]);
        p->sched_recs.push_back(make_int4(kvh, hc, kvh * group + hc * 8, std::min(8, group - hc * 8)));
      }
    }
    p->n_units = n_units;
    p->n_sched_ctas = n_units > 0 ? n_ctas : 0;
    p->sms = sms;
    p->merge_queries.clear();
    for (int i = 0; i < n_queries; ++i)
      if (p->qinfo[i].w > 1) p->merge_queries.push_back(i);
  }
  p->n_queries = n_queries;
  p->n_items = static_cast<int>(p->items.size());
  p->n_slots = slot;
  p->num_heads = num_heads;
  p->num_kv_heads = g.num_kv_heads;
  p->group = num_heads / g.num_kv_heads;
  p->n_hchunk = (p->group + 7) / 8;
  p->head_dim = g.head_dim;
  p->page_size = g.page_size;
  p->max_ctx = max_ctx;
  p->even_ctx = min_ctx == max_ctx;
  p->max_splits = max_splits;
  p->split_tokens = C;
  p->device = device;
  {
    std::vector<int32_t> r(p->rows);
    std::sort(r.begin(), r.end());
    p->rows_distinct = std::adjacent_find(r.begin(), r.end()) == r.end();
  }

  cudaError_t e;
  // Scratch (grow-only): split partials and the per-(query, head) counters.  A
  // graph-stable plan sizes the partials with the same headroom as its block, so
  // a context that adds a split does not move them (and stale the captured launches).
  const bool graph = (p->flags & KVC_PLAN_GRAPH) != 0;
  auto cap = [graph](size_t& c, size_t n) {
    if (!graph) return c = n;
    if (n > c) c = n + n / 4 + 16;
    return c;
  };
  const size_t slots = cap(p->cap_slots, static_cast<size_t>(slot));
  const size_t po_b = sizeof(float) * std::max<size_t>(1, slots * num_heads * g.head_dim);
  const size_t pml_b = sizeof(float2) * std::max<size_t>(1, slots * num_heads);
  const size_t cnt_b = sizeof(unsigned) * std::max<size_t>(1, static_cast<size_t>(n_queries) * g.num_kv_heads * p->n_hchunk);
  if ((e = p->d_part_o.ensure(po_b)) || (e = p->d_part_ml.ensure(pml_b)))
    return cuda_error(e, "plan buffers");
  const uint32_t dev_errors = g_device_errors.load();
  if (cnt_b > p->d_counters.cap || dev_errors != p->counters_zeroed_at) {
    if ((e = p->d_counters.ensure(cnt_b))) return cuda_error(e, "plan counters");
    if ((e = cudaMemsetAsync(p->d_counters.ptr, 0, p->d_counters.cap, s)))
      return cuda_error(e, "cudaMemsetAsync(counters)");
    p->counters_zeroed_at = dev_errors;
  }
  // The plan itself: one block {items | qinfo | rows | positions | unit records |
  // merge list | unit counter (zero)}, 256-byte aligned parts, staged in pinned
  // memory and uploaded with one copy.
  // A graph-stable plan lays the block out for grow-only capacities (25 % headroom),
  // so its parts keep their device addresses while rebuilds stay within them.
  auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
  const size_t items_n = sizeof(int4) * p->item_pairs.size();
  const size_t qinfo_n = sizeof(int4) * n_queries;
  const size_t rows_n = sizeof(int32_t) * n_queries;
  const size_t sched_n = sizeof(int4) * p->sched_recs.size();
  const size_t merge_n = sizeof(int32_t) * p->merge_queries.size();
  const size_t items_cap = sizeof(int4) * cap(p->cap_items, p->item_pairs.size());
  const size_t q_cap = cap(p->cap_queries, static_cast<size_t>(n_queries));
  const size_t sched_cap = sizeof(int4) * cap(p->cap_sched, p->sched_recs.size());
  // (a graph-stable plan's merge grid has a CTA per query, each of which may read
  // its slot of the list: room for every query)
  const size_t merge_cap = sizeof(int32_t) * (graph ? q_cap : cap(p->cap_merge, p->merge_queries.size()));
  const size_t o_items = 0;
  const size_t o_qinfo = o_items + al(std::max<size_t>(items_cap, 1));
  const size_t o_rows = o_qinfo + al(std::max<size_t>(sizeof(int4) * q_cap, 1));
  const size_t o_pos = o_rows + al(std::max<size_t>(sizeof(int32_t) * q_cap, 1));
  const size_t o_sched = o_pos + al(std::max<size_t>(sizeof(int32_t) * q_cap, 1));
  const size_t o_merge = o_sched + al(std::max<size_t>(sched_cap, 1));
  const size_t o_queue = o_merge + al(std::max<size_t>(merge_cap, 1));
  const size_t blob_b = o_queue + 256;
  if ((e = p->d_blob.ensure(blob_b))) return cuda_error(e, "plan buffers");
  if (p->upload_done) {  // the staging is free once the previous upload has landed
    if (const int rc = wait_event(p->upload_done, "plan upload")) return rc;
  } else if ((e = cudaEventCreateWithFlags(&p->upload_done, cudaEventDisableTiming))) {
    return cuda_error(e, "cudaEventCreate");
  }
  if ((e = p->h_stage.ensure(blob_b))) return cuda_error(e, "cudaMallocHost(plan)");
  uint8_t* h = static_cast<uint8_t*>(p->h_stage.ptr);
  if (items_n) memcpy(h + o_items, p->item_pairs.data(), items_n);
  if (qinfo_n) memcpy(h + o_qinfo, p->qinfo.data(), qinfo_n);
  if (rows_n) memcpy(h + o_rows, p->rows.data(), rows_n);
  if (rows_n) memcpy(h + o_pos, p->positions.data(), rows_n);
  if (sched_n) memcpy(h + o_sched, p->sched_recs.data(), sched_n);
  if (merge_n) memcpy(h + o_merge, p->merge_queries.data(), merge_n);
  memset(h + o_queue, 0, 256);  // the unit counter starts at zero (the merge re-arms it)
  // counts the kernels of a graph-stable plan read (64 bytes past the counter)
  int32_t* hdr = reinterpret_cast<int32_t*>(h + o_queue + 64);
  hdr[kHdrUnits] = p->n_units;
  hdr[kHdrL2Ahead] = l2_ahead_slabs(C, p->even_ctx);
  hdr[kHdrMergeQueries] = static_cast<int32_t>(p->merge_queries.size());
  hdr[kHdrMergeWph] = merge_warps_per_head(max_splits);
  if ((e = cudaMemcpyAsync(p->d_blob.ptr, h, blob_b, cudaMemcpyHostToDevice, s)))
    return cuda_error(e, "plan upload");
  uint8_t* d = static_cast<uint8_t*>(p->d_blob.ptr);
  p->dev_items = reinterpret_cast<const int4*>(d + o_items);
  p->dev_qinfo = reinterpret_cast<const int4*>(d + o_qinfo);
  p->dev_rows = reinterpret_cast<const int32_t*>(d + o_rows);
  p->dev_pos = reinterpret_cast<const int32_t*>(d + o_pos);
  p->dev_sched = reinterpret_cast<const int4*>(d + o_sched);
  p->dev_merge = reinterpret_cast<const int32_t*>(d + o_merge);
  p->dev_queue = reinterpret_cast<unsigned*>(d + o_queue);
  p->dev_hdr = reinterpret_cast<const int*>(d + o_queue + 64);
  if ((e = cudaEventRecord(p->upload_done, s))) return cuda_error(e, "cudaEventRecord(plan)");
  // what launches of this plan hold: a change makes captured launches stale
  std::vector<uintptr_t> sig = {
      reinterpret_cast<uintptr_t>(p->d_blob.ptr), o_qinfo, o_rows, o_pos, o_sched, o_merge,
      o_queue, reinterpret_cast<uintptr_t>(p->d_part_o.ptr),
      reinterpret_cast<uintptr_t>(p->d_part_ml.ptr), reinterpret_cast<uintptr_t>(p->d_counters.ptr),
      static_cast<uintptr_t>(n_queries), static_cast<uintptr_t>(num_heads),
      static_cast<uintptr_t>(g.num_kv_heads), static_cast<uintptr_t>(g.head_dim),
      static_cast<uintptr_t>(g.page_size), static_cast<uintptr_t>(g.dtype),
      static_cast<uintptr_t>(device)};
  if (sig != p->launch_sig) {
    p->launch_sig.swap(sig);
    p->generation++;
  }
  p->pool_geom = g;
  p->built_from.swap(inputs);
  p->valid = true;
  return KVC_OK;
}

int do_decode(kvc_pool* pool, const kvc_plan* plan, int layer, const void* d_q, void* d_out,
              const int32_t* d_bt, int bt_stride, float scale, cudaStream_t s) {
  return do_decode_fused(pool, plan, layer, d_q, d_out, d_bt, bt_stride, scale, nullptr, nullptr,
                         s);
}

int do_decode_fused(kvc_pool* pool, const kvc_plan* plan, int layer, const void* d_q,
                    void* d_out, const int32_t* d_bt, int bt_stride, float scale,
                    const void* d_k_new, const void* d_v_new, cudaStream_t s,
                    const XchgTarget* xt, int early) {
  const PoolGeom& g = pool->g;
  if (!plan || !plan->valid) return set_error(KVC_ERR_INVALID_ARG, "plan has not been built.");
  if (layer < 0 || layer >= g.num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for the KV pool.");
  if (plan->head_dim != g.head_dim || plan->num_kv_heads != g.num_kv_heads ||
      plan->page_size != g.page_size)
    return set_error(KVC_ERR_INVALID_ARG, "plan was built for a pool of another geometry.");
  if (plan->n_queries == 0) return KVC_OK;
  if (!d_q || (!d_out && !xt) || !d_bt)
    return set_error(KVC_ERR_INVALID_ARG, "q, out and block tables must not be null.");
  if ((reinterpret_cast<uintptr_t>(d_q) | reinterpret_cast<uintptr_t>(d_out)) & 3u)
    return set_error(KVC_ERR_INVALID_ARG, "q and out must be 4-byte aligned.");
  if (static_cast<int64_t>(plan->max_ctx) > static_cast<int64_t>(bt_stride) * g.page_size)
    return set_error(KVC_ERR_OUT_OF_RANGE, "a context length exceeds the block-table width.");
  DecodeArgs a;
  a.k_layer = pool->k + static_cast<size_t>(layer) * g.layer_bytes;
  a.v_layer = pool->v + static_cast<size_t>(layer) * g.layer_bytes;
  a.q = d_q;
  a.out = d_out;
  a.block_tables = d_bt;
  a.bt_stride = bt_stride;
  a.items = plan->dev_items;
  a.qinfo = plan->dev_qinfo;
  a.part_o = static_cast<float*>(plan->d_part_o.ptr);
  a.part_ml = static_cast<float2*>(plan->d_part_ml.ptr);
  a.counters = static_cast<unsigned*>(plan->d_counters.ptr);
  a.sched_recs = plan->dev_sched;
  a.n_units = plan->n_units;
  a.sched_cap = (plan->flags & KVC_PLAN_GRAPH) ? static_cast<int>(plan->cap_sched / 3)
                                               : plan->n_units;
  a.queue = plan->dev_queue;
  a.n_sched_ctas = plan->n_sched_ctas;
  a.early_prefetch = early >= 0 ? early : ((plan->flags & KVC_PLAN_KV_STABLE) ? 1 : 0);
  a.l2_ahead = l2_ahead_slabs(plan->split_tokens, plan->even_ctx);
  a.err_host = host_call_error_copy();
  a.merge_queries = plan->dev_merge;
  a.n_merge_queries = static_cast<int>(plan->merge_queries.size());
  a.k_new = static_cast<const uint8_t*>(d_k_new);
  a.v_new = static_cast<const uint8_t*>(d_v_new);
  a.n_items = plan->n_items;
  a.num_heads = plan->num_heads;
  a.num_kv_heads = g.num_kv_heads;
  a.group = plan->group;
  a.n_hchunk = plan->n_hchunk;
  a.head_dim = g.head_dim;
  a.page_size = g.page_size;
  a.num_pages = g.num_pages;
  a.scale_log2 = scale * kLog2e;
  a.n_queries_total = plan->n_queries;
  a.merge_wph = merge_warps_per_head(plan->max_splits);
  if ((plan->flags & KVC_PLAN_GRAPH) && plan->n_sched_ctas > 0) {
    // counts from the plan's device header; grids for any rebuild of the plan
    a.plan_hdr = plan->dev_hdr;
    a.n_sched_ctas = plan->sms * kPersistCtasPerSm;
  }
  if (xt) {
    kvc_xchg* x = xt->x;
    if (!decode_uses_mma(g.dtype, g.head_dim, g.page_size) || g.layout != kLayoutCore)
      return set_error(KVC_ERR_INVALID_ARG,
                       "a head exchange needs fp16/bf16 KV with head_dim in "
                       "{32,64,96,128,160,192,256} and a page size multiple of 16.");
    if (plan->n_units == 0) return set_error(KVC_ERR_INVALID_ARG, "empty plan in a head exchange.");
    a.xchg_peers = x->world;
    a.out_heads = xt->out_heads;
    a.out_head0 = xt->out_head0;
    for (int p = 0; p < x->world; ++p) {
      a.peer_out[p] = x->peer_base[p] + kXchgSlotsOff + static_cast<size_t>(xt->slot) * x->slot_stride;
      a.peer_flag[p] = reinterpret_cast<unsigned*>(x->peer_base[p] + kXchgFlagsOff) + x->rank;
    }
    a.epoch_ctr = reinterpret_cast<unsigned*>(x->base + kXchgEpochOff);
    a.my_flags = reinterpret_cast<const unsigned*>(x->base + kXchgFlagsOff);
    a.wait_limit_ns = x->wait_limit_ns;
  }
  cudaError_t e = launch_decode(a, g.dtype, g.layout, s);
  if (e != cudaSuccess) return cuda_error(e, "decode kernel");
  return KVC_OK;
}

int plan_queries(kvc_plan* plan, const PoolGeom& g, int q_len, int num_heads, int start_pos,
                 int kv_len, bool causal, int device, cudaStream_t s) {
  return plan_build(
      plan, g, q_len, num_heads,
      [&](int m) { return causal ? std::max(0, std::min(kv_len, start_pos + m + 1)) : kv_len; },
      [](int) { return 0; }, device, s);
}

// Decode step with one new row per query at position ctx - 1: fused into the
// attention kernel when every query has its own block-table row (a decode
// batch), else a separate append launch first (several queries of one
// sequence read each other's new rows).
int append_then_decode(kvc_pool* pool, const kvc_plan* plan, int layer, const void* d_q,
                       const void* d_k_new, const void* d_v_new, void* d_out, const int32_t* d_bt,
                       int bt_stride, float scale, cudaStream_t s, const XchgTarget* xt,
                       int early) {
  if (!d_k_new || !d_v_new) return set_error(KVC_ERR_INVALID_ARG, "K/V rows must not be null.");
  if ((reinterpret_cast<uintptr_t>(d_k_new) | reinterpret_cast<uintptr_t>(d_v_new)) & 15u)
    return set_error(KVC_ERR_INVALID_ARG, "K/V row buffers must be 16-byte aligned.");
  if (plan->rows_distinct) {
    for (int32_t c : plan->positions)
      if (c < 0) return set_error(KVC_ERR_INVALID_ARG, "a query with an empty context has no new row.");
    return do_decode_fused(pool, plan, layer, d_q, d_out, d_bt, bt_stride, scale, d_k_new, d_v_new,
                           s, xt, early);
  }
  int rc = do_append(pool, layer, d_k_new, d_v_new, d_bt, bt_stride,
                     plan->dev_rows, plan->dev_pos, 0, plan->n_queries, s);
  if (rc) return rc;
  return do_decode_fused(pool, plan, layer, d_q, d_out, d_bt, bt_stride, scale, nullptr, nullptr,
                         s, xt);
}

}  // namespace kvc

extern "C" int kvc_plan_split_tokens(const int32_t* h_ctx_lens, int n_queries, int num_heads,
                                     int num_kv_heads, int page_size, int sm_count, int* out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  if (n_queries < 0 || (n_queries > 0 && !h_ctx_lens))
    return set_error(KVC_ERR_INVALID_ARG, "ctx_lens must hold n_queries lengths.");
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be a positive multiple of num_kv_heads.");
  if (page_size <= 0 || page_size % kSlab != 0)
    return set_error(KVC_ERR_INVALID_ARG, "page_size must be a positive multiple of 16.");
  if (sm_count <= 0) return set_error(KVC_ERR_INVALID_ARG, "sm_count must be positive.");
  const int group = num_heads / num_kv_heads;
  *out = split_tokens_model(page_size, h_ctx_lens, n_queries, num_kv_heads * ((group + 7) / 8),
                            sm_count);
  return KVC_OK;
}

extern "C" int kvc_plan_split_counts(const int32_t* h_ctx_lens, int n_queries, int num_heads,
                                     int num_kv_heads, int page_size, int sm_count,
                                     int* split_tokens_out, int32_t* splits_out,
                                     int* n_splits_out) {
  if (!split_tokens_out || !n_splits_out)
    return set_error(KVC_ERR_INVALID_ARG, "split_tokens_out and n_splits_out must not be null.");
  if (n_queries < 0 || (n_queries > 0 && !h_ctx_lens))
    return set_error(KVC_ERR_INVALID_ARG, "ctx_lens must hold n_queries lengths.");
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be a positive multiple of num_kv_heads.");
  if (page_size <= 0 || page_size % kSlab != 0)
    return set_error(KVC_ERR_INVALID_ARG, "page_size must be a positive multiple of 16.");
  if (sm_count <= 0) return set_error(KVC_ERR_INVALID_ARG, "sm_count must be positive.");
  for (int i = 0; i < n_queries; ++i)
    if (h_ctx_lens[i] < 0) return set_error(KVC_ERR_INVALID_ARG, "context length must be non-negative.");
  const int group = num_heads / num_kv_heads;
  std::vector<int> refine(std::max(0, n_queries), 0);
  const int C = split_partition_sms(page_size, h_ctx_lens, n_queries,
                                    num_kv_heads * ((group + 7) / 8), sm_count, refine.data());
  int64_t total = 0;
  for (int i = 0; i < n_queries; ++i) {
    const int ns = emit_splits(i, h_ctx_lens[i], C, refine[i], [](const int4&) {});
    if (splits_out) splits_out[i] = ns;
    total += ns;
  }
  if (total > INT32_MAX) return set_error(KVC_ERR_INVALID_ARG, "too many splits.");
  *split_tokens_out = C;
  *n_splits_out = static_cast<int>(total);
  return KVC_OK;
}

extern "C" int kvc_plan_create(kvc_plan_t** out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  *out = new kvc_plan();
  return KVC_OK;
}

extern "C" int kvc_plan_destroy(kvc_plan_t* plan) {
  if (!plan) return KVC_OK;
  if (plan->device >= 0) cudaSetDevice(plan->device);
  plan->release();
  delete plan;
  return KVC_OK;
}

extern "C" int kvc_plan_decode(kvc_plan_t* plan, const kvc_pool_t* pool, const int32_t* h_rows,
                               const int32_t* h_ctx_lens, int n_queries, int num_heads,
                               void* stream) {
  if (!plan || !pool) return set_error(KVC_ERR_INVALID_ARG, "plan and pool must not be null.");
  if (n_queries > 0 && !h_ctx_lens)
    return set_error(KVC_ERR_INVALID_ARG, "ctx_lens must not be null.");
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  return plan_build(
      plan, pool->g, n_queries, num_heads, [&](int i) { return h_ctx_lens[i]; },
      [&](int i) { return h_rows ? h_rows[i] : i; }, pool->device,
      static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_plan_set_flags(kvc_plan_t* plan, int flags) {
  if (!plan) return set_error(KVC_ERR_INVALID_ARG, "plan must not be null.");
  if (flags & ~(KVC_PLAN_KV_STABLE | KVC_PLAN_GRAPH))
    return set_error(KVC_ERR_INVALID_ARG, "unknown plan flags %d.", flags);
  if ((flags ^ plan->flags) & KVC_PLAN_GRAPH) {
    // the layout rules change: the next build lays the plan out again
    plan->valid = false;
    plan->built_from.clear();
    plan->generation++;
  }
  plan->flags = flags;
  return KVC_OK;
}

extern "C" int kvc_plan_generation(const kvc_plan_t* plan, uint64_t* out) {
  if (!plan || !out) return set_error(KVC_ERR_INVALID_ARG, "plan and out must not be null.");
  *out = plan->generation;
  return KVC_OK;
}

extern "C" int kvc_plan_info(const kvc_plan_t* plan, int* n_items, int* n_ctas,
                             size_t* scratch_bytes) {
  if (!plan) return set_error(KVC_ERR_INVALID_ARG, "plan must not be null.");
  if (n_items) *n_items = plan->n_items;
  if (n_ctas) *n_ctas = plan->n_items * plan->num_kv_heads * plan->n_hchunk;
  if (scratch_bytes)
    *scratch_bytes = plan->d_part_o.cap + plan->d_part_ml.cap + plan->d_counters.cap;
  return KVC_OK;
}

extern "C" int kvc_decode(kvc_pool_t* pool, const kvc_plan_t* plan, int layer, const void* d_q,
                          void* d_out, const int32_t* d_block_tables, int bt_stride, float scale,
                          void* stream) {
  if (!pool) return set_error(KVC_ERR_INVALID_ARG, "pool must not be null.");
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  return do_decode(pool, plan, layer, d_q, d_out, d_block_tables, bt_stride, scale,
                   static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_append_decode(kvc_pool_t* pool, const kvc_plan_t* plan, int layer,
                                 const void* d_q, const void* d_k_new, const void* d_v_new,
                                 void* d_out, const int32_t* d_block_tables, int bt_stride,
                                 float scale, void* stream) {
  if (!pool || !plan) return set_error(KVC_ERR_INVALID_ARG, "pool and plan must not be null.");
  if (!plan->valid) return set_error(KVC_ERR_INVALID_ARG, "plan has not been built.");
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return append_then_decode(pool, plan, layer, d_q, d_k_new, d_v_new, d_out, d_block_tables,
                            bt_stride, scale, s);
}

// ============================================================================
// rotary position embedding (rope.hip:21-55, bindings.cpp:392-412)
// ============================================================================
namespace kvc {

void rope_inv_freq(float freq_base, int head_dim, float* out) {
  for (int i = 0; i < head_dim / 2; ++i)
    out[i] = 1.0f / std::pow(freq_base, static_cast<float>(2 * i) / static_cast<float>(head_dim));
}

int check_rope_args(int num_heads, int head_dim, float freq_base) {
  if (head_dim <= 0 || head_dim % 2 != 0)
    return set_error(KVC_ERR_INVALID_ARG, "head_dim must be a positive even integer for RoPE.");
  if (head_dim / 2 > kMaxRopePairs)
    return set_error(KVC_ERR_INVALID_ARG, "head_dim must be at most %d for RoPE.", 2 * kMaxRopePairs);
  if (num_heads < 0) return set_error(KVC_ERR_INVALID_ARG, "num_heads must be non-negative.");
  if (!(freq_base > 0.0f)) return set_error(KVC_ERR_INVALID_ARG, "freq_base must be positive.");
  return KVC_OK;
}

}  // namespace kvc

extern "C" int kvc_rope(const void* d_x, void* d_out, int n_tokens, int num_heads, int head_dim,
                        const int32_t* d_positions, int pos_offset, float freq_base, int neox,
                        int dtype, void* stream) {
  int rc = check_rope_args(num_heads, head_dim, freq_base);
  if (rc) return rc;
  if (n_tokens < 0) return set_error(KVC_ERR_INVALID_ARG, "n_tokens must be non-negative.");
  if (elem_size_of(dtype) == 0) return set_error(KVC_ERR_INVALID_ARG, "unknown dtype %d.", dtype);
  if (n_tokens == 0 || num_heads == 0) return KVC_OK;
  if (!d_x || !d_out) return set_error(KVC_ERR_INVALID_ARG, "x and out must not be null.");
  RopeArgs a = {};
  a.src[0] = static_cast<const uint8_t*>(d_x);
  a.dst[0] = static_cast<uint8_t*>(d_out);
  a.heads[0] = num_heads;
  a.heads[1] = 0;
  a.n_tokens = n_tokens;
  a.head_dim = head_dim;
  a.dtype = dtype;
  a.neox = neox ? 1 : 0;
  a.pos0 = pos_offset;
  a.positions = d_positions;
  rope_inv_freq(freq_base, head_dim, a.inv_freq);
  cudaError_t e = launch_rope(a, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_error(e, "rope kernel");
  return KVC_OK;
}

namespace {
struct RopeHostWs {
  std::mutex mu;  // one process-wide workspace, like rope.hip's RoPEWorkspace
  DevBuf buf;
};
RopeHostWs& rope_ws() {
  static RopeHostWs ws;
  return ws;
}
}  // namespace

extern "C" int kvc_rope_host(const void* h_x, void* h_out, int seq_len, int num_heads, int head_dim,
                             int pos_offset, float freq_base, int neox) {
  int rc = check_rope_args(num_heads, head_dim, freq_base);
  if (rc) return rc;
  if (seq_len < 0) return set_error(KVC_ERR_INVALID_ARG, "seq_len must be non-negative.");
  const size_t bytes = static_cast<size_t>(seq_len) * num_heads * head_dim * 2;
  if (bytes == 0) return KVC_OK;
  if (!h_x || !h_out) return set_error(KVC_ERR_INVALID_ARG, "x_in and x_out must not be null.");
  RopeHostWs& ws = rope_ws();
  std::lock_guard<std::mutex> lock(ws.mu);
  const size_t al = (bytes + 255) & ~static_cast<size_t>(255);
  cudaError_t e = ws.buf.ensure(2 * al);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(rope)");
  uint8_t* d_in = static_cast<uint8_t*>(ws.buf.ptr);
  uint8_t* d_out = d_in + al;
  cudaStream_t s = nullptr;
  if ((e = cudaMemcpyAsync(d_in, h_x, bytes, cudaMemcpyHostToDevice, s)))
    return cuda_error(e, "cudaMemcpyAsync(H2D)");
  if ((rc = kvc_rope(d_in, d_out, seq_len, num_heads, head_dim, nullptr, pos_offset, freq_base,
                     neox, KVC_DTYPE_F16, s)))
    return rc;
  return finish_host_call(s, h_out, d_out, bytes, "rope");
}

extern "C" int kvc_append_decode_rope(kvc_pool_t* pool, const kvc_plan_t* plan, int layer,
                                      const void* d_q, const void* d_k_new, const void* d_v_new,
                                      void* d_out, const int32_t* d_block_tables, int bt_stride,
                                      float scale, float freq_base, int neox, void* stream) {
  if (!pool || !plan) return set_error(KVC_ERR_INVALID_ARG, "pool and plan must not be null.");
  if (!plan->valid) return set_error(KVC_ERR_INVALID_ARG, "plan has not been built.");
  if (!d_q || !d_k_new || !d_v_new)
    return set_error(KVC_ERR_INVALID_ARG, "q and the K/V rows must not be null.");
  const PoolGeom& g = pool->g;
  int rc = check_rope_args(plan->num_heads, g.head_dim, freq_base);
  if (rc) return rc;
  if (plan->n_queries == 0) return KVC_OK;
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  kvc_plan* p = const_cast<kvc_plan*>(plan);
  const size_t n = static_cast<size_t>(plan->n_queries);
  const size_t qb = n * plan->num_heads * g.head_dim * g.elem_size;
  const size_t kb = n * g.num_kv_heads * g.head_dim * g.elem_size;
  const size_t qb_al = (qb + 255) & ~static_cast<size_t>(255);
  const size_t kb_al = (kb + 255) & ~static_cast<size_t>(255);
  cudaError_t e = p->d_rope.ensure(qb_al + kb_al);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(rope staging)");
  uint8_t* q_rot = static_cast<uint8_t*>(p->d_rope.ptr);
  uint8_t* k_rot = q_rot + qb_al;
  // q and the new K rows rotated at each query's own position (the plan's
  // positions: ctx - 1 of a decode step), then the fused append + attention.  The
  // rotation writes only this staging, so the decode behind it may stream KV
  // while it runs.
  RopeArgs a = {};
  a.src[0] = static_cast<const uint8_t*>(d_q);
  a.dst[0] = q_rot;
  a.heads[0] = plan->num_heads;
  a.src[1] = static_cast<const uint8_t*>(d_k_new);
  a.dst[1] = k_rot;
  a.heads[1] = g.num_kv_heads;
  a.n_tokens = plan->n_queries;
  a.head_dim = g.head_dim;
  a.dtype = g.dtype;
  a.neox = neox ? 1 : 0;
  a.positions = plan->dev_pos;
  rope_inv_freq(freq_base, g.head_dim, a.inv_freq);
  if ((e = launch_rope(a, s, true)) != cudaSuccess) return cuda_error(e, "rope kernel");
  return append_then_decode(pool, plan, layer, q_rot, k_rot, d_v_new, d_out, d_block_tables,
                            bt_stride, scale, s, nullptr, 1);
}

extern "C" int kvc_decode_host(kvc_pool_t* pool, const kvc_plan_t* plan, int layer,
                               const void* h_q, const void* h_k_new, const void* h_v_new,
                               void* h_out, const int32_t* d_block_tables, int bt_stride,
                               float scale, void* stream) {
  if (!pool || !plan) return set_error(KVC_ERR_INVALID_ARG, "pool and plan must not be null.");
  if (!plan->valid) return set_error(KVC_ERR_INVALID_ARG, "plan has not been built.");
  if (!h_q || !h_k_new || !h_v_new || !h_out)
    return set_error(KVC_ERR_INVALID_ARG, "host buffers must not be null.");
  const PoolGeom& g = pool->g;
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t n = static_cast<size_t>(plan->n_queries);
  const size_t qb = n * plan->num_heads * g.head_dim * g.elem_size;
  const size_t kb = n * g.num_kv_heads * g.head_dim * g.elem_size;
  const size_t kb_al = (kb + 255) & ~static_cast<size_t>(255);
  const size_t qb_al = (qb + 255) & ~static_cast<size_t>(255);
  cudaError_t e = pool->io.ensure(qb_al + 2 * kb_al);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(io)");
  uint8_t* d = static_cast<uint8_t*>(pool->io.ptr);
  uint8_t* const d_in[3] = {d, d + qb_al, d + qb_al + kb_al};  // q, new K rows, new V rows
  // Inputs reach the device through the staging kernel (it writes no pages or
  // block tables, so the decode behind it may start streaming KV early).
  const void* h_in[3] = {h_q, h_k_new, h_v_new};
  const size_t in_b[3] = {qb, kb, kb};
  HostCallStage st;
  int rc = stage_host_call(pool->io_host, h_in, in_b, d_in, h_out, qb, s, &st);
  if (rc) return rc;
  rc = append_then_decode(pool, plan, layer, d_in[0], d_in[1], d_in[2], st.out_dev, d_block_tables,
                          bt_stride, scale, s, nullptr, 1);
  if (rc) return rc;
  return finish_staged_call(s, h_out, st, qb, "kvc_decode_host",
                            decode_uses_mma(g.dtype, g.head_dim, g.page_size));
}

// ============================================================================
// reference-compatible process-wide pool (DeviceKVCachePool, attention.hip:168-224)
// ============================================================================
namespace {

struct Singleton {
  std::mutex mu;             // bindings.cpp:18 (g_hip_workspace_mutex)
  kvc_pool pool;             // paged pool, one sequence, identity block table
  bool live = false;
  int max_seq_len = 0;
  DevBuf bt;                 // identity block table
  int bt_len = 0;
  kvc_plan plan;
  cudaStream_t stream = nullptr;
  int stream_device = -1;
  DevBuf layer_ws;           // intermediates of forward_layer_cached
  DevBuf layer_io;           // its host inputs (activations, norms, weights) on the device
};

Singleton& singleton() {
  static Singleton s;
  return s;
}

// Scratch context of the full-KV host entry point (launch_gqa_attention_fp16,
// attention.hip:228-284 keeps an AttentionWorkspace for the same purpose).
struct HostAttnCtx {
  kvc_pool pool;
  DevBuf bt;
  int bt_len = 0;
  DevBuf bounce;
  kvc_plan plan;
  cudaStream_t stream = nullptr;
  int stream_device = -1;
};

HostAttnCtx& host_attn_ctx() {
  static HostAttnCtx c;
  return c;
}

int ensure_stream(cudaStream_t* s, int* s_dev, int device) {
  if (*s && *s_dev == device) return KVC_OK;
  cudaError_t e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_error(e, "cudaStreamCreate");
  *s_dev = device;
  return KVC_OK;
}

int ensure_identity_table(DevBuf* bt, int* bt_len, int pages, cudaStream_t s) {
  if (pages <= *bt_len) return KVC_OK;
  cudaError_t e = bt->ensure(sizeof(int32_t) * pages);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(block table)");
  std::vector<int32_t> ids(pages);
  for (int i = 0; i < pages; ++i) ids[i] = i;
  if ((e = cudaMemcpyAsync(bt->ptr, ids.data(), sizeof(int32_t) * pages, cudaMemcpyHostToDevice, s)))
    return cuda_error(e, "cudaMemcpy(block table)");
  if (const int rc = wait_stream(s, "block table upload")) return rc;
  *bt_len = pages;
  return KVC_OK;
}

constexpr int kDefaultPageSize = 16;

int cache_init_locked(Singleton& S, int num_layers, int max_seq_len, int num_kv_heads,
                      int head_dim, int dtype, int page_size) {
  if (num_layers <= 0 || max_seq_len <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return set_error(KVC_ERR_INVALID_ARG, "KV cache dimensions must all be positive.");
  if (page_size == 0) page_size = kDefaultPageSize;
  const int pages = (max_seq_len + page_size - 1) / page_size;
  PoolGeom g;
  int rc = make_geom(num_layers, pages, page_size, num_kv_heads, head_dim, dtype, &g);
  if (rc) return rc;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if ((rc = ensure_stream(&S.stream, &S.stream_device, device))) return rc;
  if ((rc = pool_alloc(&S.pool, g, device))) {
    S.live = false;
    return rc;
  }
  if ((rc = ensure_identity_table(&S.bt, &S.bt_len, pages, S.stream))) {
    S.live = false;
    return rc;
  }
  S.max_seq_len = max_seq_len;
  S.live = true;
  return KVC_OK;
}

// Validation of attention.hip:316-329, in the same order and with the same classes.
int validate_cached(const Singleton& S, int layer_idx, int q_len, int start_pos, int num_heads,
                    int num_kv_heads, int head_dim) {
  if (!S.live)
    return set_error(KVC_ERR_RUNTIME, "Device KV cache not initialized. Call kv_cache_init first.");
  if (layer_idx < 0 || layer_idx >= S.pool.g.num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for DeviceKVCachePool.");
  const int64_t kv_len = static_cast<int64_t>(start_pos) + q_len;
  if (start_pos < 0 || kv_len > S.max_seq_len)
    return set_error(KVC_ERR_OUT_OF_RANGE,
                     "start_pos + q_len exceeds max_seq_len in DeviceKVCachePool.");
  if (num_kv_heads != S.pool.g.num_kv_heads || head_dim != S.pool.g.head_dim)
    return set_error(KVC_ERR_INVALID_ARG,
                     "num_kv_heads or head_dim mismatch with DeviceKVCachePool.");
  if (num_heads <= 0 || num_heads % num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be divisible by num_kv_heads.");
  if (q_len < 0) return set_error(KVC_ERR_INVALID_ARG, "q_len must be non-negative.");
  return KVC_OK;
}

}  // namespace

namespace kvc {

int cached_plan(kvc_pool* pool, kvc_plan* plan, int q_len, int start_pos, int num_heads,
                bool causal, cudaStream_t s) {
  return plan_queries(plan, pool->g, q_len, num_heads, start_pos, start_pos + q_len, causal,
                      pool->device, s);
}

int cached_run(kvc_pool* pool, const kvc_plan* plan, const int32_t* d_bt, int bt_len,
               const void* d_Q, const void* d_Kn, const void* d_Vn, void* d_Out, int layer_idx,
               int q_len, int start_pos, float scale, cudaStream_t s, int early) {
  if (q_len == 1)  // a decode step: the row append runs inside the attention kernel
    return append_then_decode(pool, plan, layer_idx, d_Q, d_Kn, d_Vn, d_Out, d_bt, bt_len, scale,
                              s, nullptr, early);
  int rc =
      do_append(pool, layer_idx, d_Kn, d_Vn, d_bt, bt_len, nullptr, nullptr, start_pos, q_len, s);
  if (rc) return rc;
  return do_decode(pool, plan, layer_idx, d_Q, d_Out, d_bt, bt_len, scale, s);
}

}  // namespace kvc

extern "C" int kvc_cache_init(int num_layers, int max_seq_len, int num_kv_heads, int head_dim) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  return cache_init_locked(S, num_layers, max_seq_len, num_kv_heads, head_dim, KVC_DTYPE_F16,
                           kDefaultPageSize);
}

extern "C" int kvc_cache_init_ex(int num_layers, int max_seq_len, int num_kv_heads, int head_dim,
                                 int dtype, int page_size) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  return cache_init_locked(S, num_layers, max_seq_len, num_kv_heads, head_dim, dtype, page_size);
}

extern "C" int kvc_cache_free(void) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  if (S.pool.k || S.pool.v) {
    cudaSetDevice(S.pool.device);
    pool_release(&S.pool);
    S.layer_ws.release();
    S.layer_io.release();
  }
  S.live = false;
  S.max_seq_len = 0;
  return KVC_OK;
}

extern "C" int kvc_cache_dtype(void) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  return S.live ? S.pool.g.dtype : -1;
}

extern "C" int kvc_gqa_attention_cached(const void* h_Q, const void* h_K_new,
                                        const void* h_V_new, void* h_Out, int layer_idx,
                                        int q_len, int start_pos, int num_heads,
                                        int num_kv_heads, int head_dim, float scale,
                                        int causal) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  int rc = validate_cached(S, layer_idx, q_len, start_pos, num_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (q_len == 0) return KVC_OK;
  if (!h_Q || !h_K_new || !h_V_new || !h_Out)
    return set_error(KVC_ERR_INVALID_ARG, "host buffers must not be null.");
  if (const int rc_dev = use_device(S.pool.device)) return rc_dev;
  const PoolGeom& g = S.pool.g;
  const size_t qb = static_cast<size_t>(q_len) * num_heads * head_dim * g.elem_size;
  const size_t kb = static_cast<size_t>(q_len) * num_kv_heads * head_dim * g.elem_size;
  const size_t qb_al = (qb + 255) & ~static_cast<size_t>(255);
  const size_t kb_al = (kb + 255) & ~static_cast<size_t>(255);
  cudaError_t e = S.pool.io.ensure(qb_al + 2 * kb_al);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(io)");
  uint8_t* d = static_cast<uint8_t*>(S.pool.io.ptr);
  uint8_t* const d_in[3] = {d, d + qb_al, d + qb_al + kb_al};  // q, new K rows, new V rows
  cudaStream_t s = S.stream;
  if ((rc = cached_plan(&S.pool, &S.plan, q_len, start_pos, num_heads, causal != 0, s))) return rc;
  const void* h_in[3] = {h_Q, h_K_new, h_V_new};
  const size_t in_b[3] = {qb, kb, kb};
  HostCallStage st;
  if ((rc = stage_host_call(S.pool.io_host, h_in, in_b, d_in, h_Out, qb, s, &st))) return rc;
  rc = cached_run(&S.pool, &S.plan, static_cast<const int32_t*>(S.bt.ptr), S.bt_len, d_in[0],
                  d_in[1], d_in[2], st.out_dev, layer_idx, q_len, start_pos, scale, s, 1);
  if (rc) return rc;
  return finish_staged_call(s, h_Out, st, qb, "gqa_attention_cached",
                            decode_uses_mma(g.dtype, g.head_dim, g.page_size));
}

extern "C" int kvc_gqa_attention_cached_device(const void* d_Q, const void* d_K_new,
                                               const void* d_V_new, void* d_Out, int layer_idx,
                                               int q_len, int start_pos, int num_heads,
                                               int num_kv_heads, int head_dim, float scale,
                                               int causal, void* stream) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  int rc = validate_cached(S, layer_idx, q_len, start_pos, num_heads, num_kv_heads, head_dim);
  if (rc) return rc;
  if (q_len == 0) return KVC_OK;
  if (const int rc_dev = use_device(S.pool.device)) return rc_dev;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = cached_plan(&S.pool, &S.plan, q_len, start_pos, num_heads, causal != 0, s))) return rc;
  return cached_run(&S.pool, &S.plan, static_cast<const int32_t*>(S.bt.ptr), S.bt_len, d_Q,
                    d_K_new, d_V_new, d_Out, layer_idx, q_len, start_pos, scale, s, -1);
}

namespace {

LayerDims layer_dims(int layer_idx, int seq_len, int pos_offset, int hidden_size,
                     int intermediate_size, int num_heads, int num_kv_heads, int head_dim,
                     float rms_norm_eps, float rope_freq_base, int rope_neox, float scale) {
  LayerDims d;
  d.layer = layer_idx;
  d.seq = seq_len;
  d.pos = pos_offset;
  d.hidden = hidden_size;
  d.inter = intermediate_size;
  d.H = num_heads;
  d.Hkv = num_kv_heads;
  d.D = head_dim;
  d.eps = rms_norm_eps;
  d.base = rope_freq_base;
  d.scale = scale;
  d.neox = rope_neox != 0;
  return d;
}

}  // namespace

extern "C" int kvc_forward_layer_cached(
    const void* h_x_in, void* h_x_out, const void* h_attn_norm_w, const void* h_wq, int wq_type,
    const void* h_wk, int wk_type, const void* h_wv, int wv_type, const void* h_wo, int wo_type,
    const void* h_ffn_norm_w, const void* h_wgate, int wgate_type, const void* h_wup,
    int wup_type, const void* h_wdown, int wdown_type, int layer_idx, int seq_len, int pos_offset,
    int hidden_size, int intermediate_size, int num_heads, int num_kv_heads, int head_dim,
    float rms_norm_eps, float rope_freq_base, int rope_neox, float scale) {
  const LayerDims d = layer_dims(layer_idx, seq_len, pos_offset, hidden_size, intermediate_size,
                                 num_heads, num_kv_heads, head_dim, rms_norm_eps, rope_freq_base,
                                 rope_neox, scale);
  const int types[7] = {wq_type, wk_type, wv_type, wo_type, wgate_type, wup_type, wdown_type};
  const void* h_w[7] = {h_wq, h_wk, h_wv, h_wo, h_wgate, h_wup, h_wdown};
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  int rc = check_layer(d, types);
  if (rc) return rc;
  if ((rc = validate_cached(S, layer_idx, seq_len, pos_offset, num_heads, num_kv_heads, head_dim)))
    return rc;
  if (seq_len == 0) return KVC_OK;
  if (!h_x_in || !h_x_out || !h_attn_norm_w || !h_ffn_norm_w)
    return set_error(KVC_ERR_INVALID_ARG, "host buffers must not be null.");
  for (const void* w : h_w)
    if (!w) return set_error(KVC_ERR_INVALID_ARG, "weight buffers must not be null.");
  if (const int rc_dev = use_device(S.pool.device)) return rc_dev;
  cudaStream_t s = S.stream;
  // attention.hip:629-644: the activations, the norm weights and every weight are
  // copied to the device on each call; everything in between stays there.
  auto al = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
  const size_t xb = sizeof(uint16_t) * static_cast<size_t>(seq_len) * hidden_size;
  const size_t nb = sizeof(uint16_t) * static_cast<size_t>(hidden_size);
  size_t wb[7];
  const size_t wtot = layer_weight_bytes(d, types, wb);
  cudaError_t e = S.layer_io.ensure(2 * al(xb) + 2 * al(nb) + wtot);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(layer inputs)");
  uint8_t* p = static_cast<uint8_t*>(S.layer_io.ptr);
  LayerIO io;
  uint8_t* d_x = p;
  uint8_t* d_out = p + al(xb);
  uint8_t* d_an = d_out + al(xb);
  uint8_t* d_fn = d_an + al(nb);
  uint8_t* d_w = d_fn + al(nb);
  if ((e = cudaMemcpyAsync(d_x, h_x_in, xb, cudaMemcpyHostToDevice, s)) ||
      (e = cudaMemcpyAsync(d_an, h_attn_norm_w, nb, cudaMemcpyHostToDevice, s)) ||
      (e = cudaMemcpyAsync(d_fn, h_ffn_norm_w, nb, cudaMemcpyHostToDevice, s)))
    return cuda_error(e, "cudaMemcpyAsync(layer inputs)");
  for (int i = 0; i < 7; ++i) {
    if ((e = cudaMemcpyAsync(d_w, h_w[i], wb[i], cudaMemcpyHostToDevice, s)))
      return cuda_error(e, "cudaMemcpyAsync(weights)");
    io.w[i] = d_w;
    io.type[i] = types[i];
    d_w += al(wb[i]);
  }
  io.x_in = reinterpret_cast<const __half*>(d_x);
  io.x_out = reinterpret_cast<__half*>(d_out);
  io.attn_norm = reinterpret_cast<const __half*>(d_an);
  io.ffn_norm = reinterpret_cast<const __half*>(d_fn);
  rc = layer_forward(&S.pool, &S.plan, static_cast<const int32_t*>(S.bt.ptr), S.bt_len,
                     S.layer_ws, io, d, s);
  if (rc) return rc;
  return finish_host_call(s, h_x_out, d_out, xb, "forward_layer_cached");
}

extern "C" int kvc_forward_layer_cached_device(
    const void* d_x_in, void* d_x_out, const void* d_attn_norm_w, const void* d_wq, int wq_type,
    const void* d_wk, int wk_type, const void* d_wv, int wv_type, const void* d_wo, int wo_type,
    const void* d_ffn_norm_w, const void* d_wgate, int wgate_type, const void* d_wup,
    int wup_type, const void* d_wdown, int wdown_type, int layer_idx, int seq_len, int pos_offset,
    int hidden_size, int intermediate_size, int num_heads, int num_kv_heads, int head_dim,
    float rms_norm_eps, float rope_freq_base, int rope_neox, float scale, void* stream) {
  const LayerDims d = layer_dims(layer_idx, seq_len, pos_offset, hidden_size, intermediate_size,
                                 num_heads, num_kv_heads, head_dim, rms_norm_eps, rope_freq_base,
                                 rope_neox, scale);
  LayerIO io;
  const int types[7] = {wq_type, wk_type, wv_type, wo_type, wgate_type, wup_type, wdown_type};
  const void* w[7] = {d_wq, d_wk, d_wv, d_wo, d_wgate, d_wup, d_wdown};
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  int rc = check_layer(d, types);
  if (rc) return rc;
  if ((rc = validate_cached(S, layer_idx, seq_len, pos_offset, num_heads, num_kv_heads, head_dim)))
    return rc;
  if (seq_len == 0) return KVC_OK;
  if (!d_x_in || !d_x_out || !d_attn_norm_w || !d_ffn_norm_w)
    return set_error(KVC_ERR_INVALID_ARG, "device buffers must not be null.");
  for (int i = 0; i < 7; ++i) {
    if (!w[i]) return set_error(KVC_ERR_INVALID_ARG, "weight buffers must not be null.");
    io.w[i] = w[i];
    io.type[i] = types[i];
  }
  io.x_in = static_cast<const __half*>(d_x_in);
  io.x_out = static_cast<__half*>(d_x_out);
  io.attn_norm = static_cast<const __half*>(d_attn_norm_w);
  io.ffn_norm = static_cast<const __half*>(d_ffn_norm_w);
  if (const int rc_dev = use_device(S.pool.device)) return rc_dev;
  return layer_forward(&S.pool, &S.plan, static_cast<const int32_t*>(S.bt.ptr), S.bt_len,
                       S.layer_ws, io, d, static_cast<cudaStream_t>(stream));
}

extern "C" int kvc_cache_gather(int layer_idx, int start, int count, void* h_K_out,
                                void* h_V_out) {
  Singleton& S = singleton();
  std::lock_guard<std::mutex> lock(S.mu);
  if (!S.live)
    return set_error(KVC_ERR_RUNTIME, "Device KV cache not initialized. Call kv_cache_init first.");
  if (layer_idx < 0 || layer_idx >= S.pool.g.num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for DeviceKVCachePool.");
  if (start < 0 || count < 0 || static_cast<int64_t>(start) + count > S.max_seq_len)
    return set_error(KVC_ERR_OUT_OF_RANGE, "gather range exceeds max_seq_len.");
  if (count == 0) return KVC_OK;
  if (!h_K_out || !h_V_out) return set_error(KVC_ERR_INVALID_ARG, "outputs must not be null.");
  if (const int rc_dev = use_device(S.pool.device)) return rc_dev;
  const PoolGeom& g = S.pool.g;
  const size_t rb = static_cast<size_t>(count) * g.num_kv_heads * g.head_dim * g.elem_size;
  const size_t rb_al = (rb + 255) & ~static_cast<size_t>(255);
  cudaError_t e = S.pool.io.ensure(2 * rb_al);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(io)");
  uint8_t* d = static_cast<uint8_t*>(S.pool.io.ptr);
  cudaStream_t s = S.stream;
  int rc = kvc_gather(&S.pool, layer_idx, static_cast<const int32_t*>(S.bt.ptr), S.bt_len, 0,
                      start, count, d, d + rb_al, s);
  if (rc) return rc;
  if ((e = cudaMemcpyAsync(h_K_out, d, rb, cudaMemcpyDeviceToHost, s)) ||
      (e = cudaMemcpyAsync(h_V_out, d + rb_al, rb, cudaMemcpyDeviceToHost, s)))
    return cuda_error(e, "cudaMemcpyAsync(D2H)");
  return finish_host_call(s, nullptr, nullptr, 0, "kv_cache_gather");
}

// Full-KV host attention (launch_gqa_attention_fp16, attention.hip:228-284): the
// layer's K/V rows come from host memory on every call.  They are copied to a
// device bounce buffer, scattered into a one-layer scratch pool with the same
// page geometry as the resident pool and attended by the same kernels, so the
// result is bit-identical to the resident path for the same rows.
extern "C" int kvc_gqa_attention_ex(const void* h_Q, const void* h_K, const void* h_V,
                                    void* h_Out, int q_len, int kv_len, int num_heads,
                                    int num_kv_heads, int head_dim, int start_pos, float scale,
                                    int causal, int dtype) {
  // attention.hip:242-247
  if (head_dim <= 0 || head_dim > 256)
    return set_error(KVC_ERR_INVALID_ARG, "head_dim must be in (0, 256] for gqa_attention.");
  if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be divisible by num_kv_heads.");
  if (num_heads <= 0) return set_error(KVC_ERR_INVALID_ARG, "num_heads must be positive.");
  if (q_len < 0 || kv_len < 0)
    return set_error(KVC_ERR_INVALID_ARG, "q_len and kv_len must be non-negative.");
  const int es = elem_size_of(dtype);
  if (es == 0) return set_error(KVC_ERR_INVALID_ARG, "unsupported KV storage dtype %d.", dtype);
  if (q_len == 0) return KVC_OK;
  if (!h_Q || !h_Out || (kv_len > 0 && (!h_K || !h_V)))
    return set_error(KVC_ERR_INVALID_ARG, "host buffers must not be null.");

  Singleton& S = singleton();  // one process-wide mutex, as bindings.cpp:18
  std::lock_guard<std::mutex> lock(S.mu);
  HostAttnCtx& C = host_attn_ctx();
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  int rc = ensure_stream(&C.stream, &C.stream_device, device);
  if (rc) return rc;
  const int pages = std::max(1, (kv_len + kDefaultPageSize - 1) / kDefaultPageSize);
  PoolGeom g;
  if ((rc = make_geom(1, pages, kDefaultPageSize, num_kv_heads, head_dim, dtype, &g))) return rc;
  if ((rc = pool_alloc(&C.pool, g, device))) return rc;
  if ((rc = ensure_identity_table(&C.bt, &C.bt_len, pages, C.stream))) return rc;
  cudaStream_t s = C.stream;
  const size_t kvb = static_cast<size_t>(kv_len) * num_kv_heads * head_dim * es;
  const size_t qb = static_cast<size_t>(q_len) * num_heads * head_dim * es;
  const size_t kvb_al = (kvb + 255) & ~static_cast<size_t>(255);
  const size_t qb_al = (qb + 255) & ~static_cast<size_t>(255);
  if ((e = C.bounce.ensure(2 * kvb_al + qb_al))) return cuda_error(e, "cudaMalloc(bounce)");
  uint8_t* d = static_cast<uint8_t*>(C.bounce.ptr);
  uint8_t *d_k = d, *d_v = d + kvb_al, *d_q = d + 2 * kvb_al;
  // the whole K/V crosses on the copy engine; q and the output like the cached call
  if (kvb > 0 && ((e = cudaMemcpyAsync(d_k, h_K, kvb, cudaMemcpyHostToDevice, s)) ||
                  (e = cudaMemcpyAsync(d_v, h_V, kvb, cudaMemcpyHostToDevice, s))))
    return cuda_error(e, "cudaMemcpyAsync(H2D K/V)");
  const int32_t* bt = static_cast<const int32_t*>(C.bt.ptr);
  if ((rc = do_append(&C.pool, 0, d_k, d_v, bt, C.bt_len, nullptr, nullptr, 0, kv_len, s)))
    return rc;
  rc = plan_queries(&C.plan, g, q_len, num_heads, start_pos, kv_len, causal != 0, device, s);
  if (rc) return rc;
  const void* h_in[3] = {h_Q, nullptr, nullptr};
  const size_t in_b[3] = {qb, 0, 0};
  uint8_t* const d_in[3] = {d_q, nullptr, nullptr};
  HostCallStage st;
  if ((rc = stage_host_call(C.pool.io_host, h_in, in_b, d_in, h_Out, qb, s, &st))) return rc;
  if ((rc = do_decode(&C.pool, &C.plan, 0, d_q, st.out_dev, bt, C.bt_len, scale, s))) return rc;
  return finish_staged_call(s, h_Out, st, qb, "gqa_attention",
                            decode_uses_mma(g.dtype, g.head_dim, g.page_size));
}

extern "C" int kvc_gqa_attention(const void* h_Q, const void* h_K, const void* h_V, void* h_Out,
                                 int q_len, int kv_len, int num_heads, int num_kv_heads,
                                 int head_dim, int start_pos, float scale, int causal) {
  return kvc_gqa_attention_ex(h_Q, h_K, h_V, h_Out, q_len, kv_len, num_heads, num_kv_heads,
                              head_dim, start_pos, scale, causal, KVC_DTYPE_F16);
}

extern "C" int kvc_host_alloc(size_t bytes, void** out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  *out = nullptr;
  if (bytes == 0) return set_error(KVC_ERR_INVALID_ARG, "bytes must be positive.");
  cudaError_t e = host_alloc(out, bytes, cudaHostAllocPortable);
  if (e != cudaSuccess) {
    *out = nullptr;
    return cuda_error(e, "cudaHostAlloc");
  }
  return KVC_OK;
}

extern "C" int kvc_host_free(void* ptr) {
  if (!ptr) return KVC_OK;
  cudaError_t e = cudaFreeHost(ptr);
  if (e != cudaSuccess) return cuda_error(e, "cudaFreeHost");
  return KVC_OK;
}
