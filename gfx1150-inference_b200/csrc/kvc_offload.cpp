// Host-streamed KV offload: the --offload-kv-cpu / --kv-mmap-dir modes of
// gfx1150-inference (src/kv_cache.py:100-135, :219-239, src/inference.py:518-519).
//
// The reference keeps K/V in host arrays (num_layers, max_seq_len, Hkv, D) and,
// for every layer of every step, copies the layer's whole [0, kv_len) K and V
// synchronously from pageable memory before attending (attention.hip:255-257).
// Here the host arrays are page-locked (allocated pinned, or registered), and
//   copy stream:    H2D of a layer's rows into one of two device bounce buffers
//   compute stream: scatter bounce -> one-layer paged pool (the append kernel),
//                   split-K attention (the resident path's kernels), D2H out
// run concurrently: while layer L attends, the copy engine already streams
// layer L+1 (the rows of the cached prefix, which are final) into the other
// bounce buffer.  The attention itself is the resident path's code on the same
// page geometry and split partition, so outputs are bit-identical to the
// GPU-resident pool's.
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "kvcache.h"
#include "kvc_common.h"
#include "kvc_internal.h"

using namespace kvc;

namespace {
constexpr int kOffloadPageSize = 16;  // same page geometry as the resident pool
constexpr int kTimingRing = 64;
}  // namespace

struct kvc_offload {
  std::mutex mu;
  int device = 0;
  int num_layers = 0, max_seq_len = 0, num_kv_heads = 0, head_dim = 0, dtype = 0, es = 0;
  size_t row_bytes = 0;     // num_kv_heads * head_dim * es
  size_t layer_bytes = 0;   // max_seq_len * row_bytes (host)
  uint8_t* h_k = nullptr;
  uint8_t* h_v = nullptr;
  bool registered = false;  // this object registered h_k / h_v (unregister on destroy)
  bool dma_ok = false;      // host pools are page-locked

  kvc_pool slot;            // one-layer paged pool the attention reads
  DevBuf bt;                // identity block table of the slot
  int bt_len = 0;
  kvc_plan plan;
  DevBuf io;                // q device staging
  HostBuf io_host;          // page-locked staging of pageable q / out

  struct Bounce {
    DevBuf k, v;            // token-major rows of one layer
    int layer = -1;         // layer whose rows [0, rows) are (being) copied here
    int rows = 0;
    cudaEvent_t ready = nullptr;  // copy stream: rows have landed
    cudaEvent_t free = nullptr;   // compute stream: last reader (scatter) finished
  } b[2];
  int last_used = 1;        // bounce used by the latest attend

  cudaStream_t copy = nullptr, compute = nullptr;

  // HBM mirror of layers [0, n_mirror) (kvc_offload_set_mirror): their pages stay
  // on the device; an attend uploads only the rows the mirror lacks.
  kvc_pool mirror;
  int n_mirror = 0;
  std::vector<int> mirror_rows;  // rows [0, mirror_rows[l]) of layer l are current
  DevBuf mstage_k, mstage_v;     // H2D staging of mirror uploads

  // copy-engine timing: ring of (start, stop, bytes) harvested when complete
  cudaEvent_t t_start[kTimingRing] = {}, t_stop[kTimingRing] = {};
  double t_bytes[kTimingRing] = {};
  int t_head = 0, t_tail = 0;

  double h2d_bytes = 0.0, h2d_ms = 0.0;  // streamed layers (copy-stream events)
  double mirror_bytes = 0.0;             // rows uploaded into the HBM mirror
  int64_t hits = 0, calls = 0;
};

namespace {

// Add up the copy-engine time of completed copies; wait (bounded) for the ones in
// flight when `wait`.
int harvest(kvc_offload* o, bool wait) {
  while (o->t_tail != o->t_head) {
    const int i = o->t_tail % kTimingRing;
    if (wait) {
      if (const int rc = wait_event(o->t_stop[i], "offload copy")) return rc;
    } else if (cudaEventQuery(o->t_stop[i]) != cudaSuccess) {
      cudaGetLastError();  // cudaErrorNotReady is not an error of the next call
      break;
    }
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, o->t_start[i], o->t_stop[i]) == cudaSuccess) o->h2d_ms += ms;
    o->t_tail++;
  }
  return KVC_OK;
}

// H2D of rows [r0, r1) of `layer` into bounce `bi`, on the copy stream.
int copy_rows(kvc_offload* o, int bi, int layer, int r0, int r1) {
  if (r1 <= r0) return KVC_OK;
  kvc_offload::Bounce& B = o->b[bi];
  const size_t off = static_cast<size_t>(r0) * o->row_bytes;
  const size_t n = static_cast<size_t>(r1 - r0) * o->row_bytes;
  const uint8_t* hk = o->h_k + static_cast<size_t>(layer) * o->layer_bytes + off;
  const uint8_t* hv = o->h_v + static_cast<size_t>(layer) * o->layer_bytes + off;
  if (o->t_head - o->t_tail >= kTimingRing) {
    if (const int rc = harvest(o, true)) return rc;
  }
  const int ti = o->t_head % kTimingRing;
  cudaError_t e;
  if ((e = cudaEventRecord(o->t_start[ti], o->copy)) ||
      (e = cudaMemcpyAsync(static_cast<uint8_t*>(B.k.ptr) + off, hk, n, cudaMemcpyHostToDevice, o->copy)) ||
      (e = cudaMemcpyAsync(static_cast<uint8_t*>(B.v.ptr) + off, hv, n, cudaMemcpyHostToDevice, o->copy)) ||
      (e = cudaEventRecord(o->t_stop[ti], o->copy)))
    return cuda_error(e, "offload H2D");
  o->t_bytes[ti] = 2.0 * static_cast<double>(n);
  o->t_head++;
  o->h2d_bytes += 2.0 * static_cast<double>(n);
  return KVC_OK;
}

// Start filling bounce `bi` with rows [0, rows) of `layer`.
int start_fill(kvc_offload* o, int bi, int layer, int rows) {
  kvc_offload::Bounce& B = o->b[bi];
  cudaError_t e = cudaStreamWaitEvent(o->copy, B.free, 0);  // its last reader is done
  if (e != cudaSuccess) return cuda_error(e, "cudaStreamWaitEvent(copy)");
  B.layer = layer;
  B.rows = 0;
  int rc = copy_rows(o, bi, layer, 0, rows);
  if (rc) return rc;
  B.rows = rows;
  if ((e = cudaEventRecord(B.ready, o->copy))) return cuda_error(e, "cudaEventRecord(ready)");
  return KVC_OK;
}

// Waits (bounded) for the engine's streams, then frees everything.  When a wait
// runs out nothing is freed (the GPU may still use it) and the status says so.
int destroy_locked(kvc_offload* o) {
  cudaSetDevice(o->device);
  int rc = KVC_OK;
  if (o->copy && (rc = wait_stream(o->copy, "offload copy stream"))) return rc;
  if (o->compute && (rc = wait_stream(o->compute, "offload compute stream"))) return rc;
  for (auto& B : o->b) {
    B.k.release();
    B.v.release();
    if (B.ready) cudaEventDestroy(B.ready);
    if (B.free) cudaEventDestroy(B.free);
    B.ready = B.free = nullptr;
  }
  for (int i = 0; i < kTimingRing; ++i) {
    if (o->t_start[i]) cudaEventDestroy(o->t_start[i]);
    if (o->t_stop[i]) cudaEventDestroy(o->t_stop[i]);
    o->t_start[i] = o->t_stop[i] = nullptr;
  }
  pool_release(&o->slot);
  pool_release(&o->mirror);
  o->n_mirror = 0;
  o->mirror_rows.clear();
  o->mstage_k.release();
  o->mstage_v.release();
  o->bt.release();
  o->io.release();
  o->io_host.release();
  o->plan.release();
  if (o->registered) {
    cudaHostUnregister(o->h_k);
    cudaHostUnregister(o->h_v);
    o->registered = false;
  }
  if (o->copy) cudaStreamDestroy(o->copy);
  if (o->compute) cudaStreamDestroy(o->compute);
  o->copy = o->compute = nullptr;
  return KVC_OK;
}

}  // namespace

namespace {

// The query reaches d_q through the input staging kernel; the output goes where
// stage_host_call puts it (the host buffer itself when page-locked).
int stage_q(kvc_offload* o, const void* h_Q, uint8_t* d_q, size_t qb, void* h_Out, cudaStream_t s,
            HostCallStage* st) {
  const void* h_in[3] = {h_Q, nullptr, nullptr};
  const size_t in_b[3] = {qb, 0, 0};
  uint8_t* const d_in[3] = {d_q, nullptr, nullptr};
  return stage_host_call(o->io_host, h_in, in_b, d_in, h_Out, qb, s, st);
}

// The next layer after `layer` that is streamed (not mirrored), cyclically, and
// how many of its rows are final now: within a step the prefix [0, start_pos);
// a layer of the next step [0, total).  Prefetch it into bounce `bi` unless a
// bounce already holds it.
int prefetch_next(kvc_offload* o, int layer, int start_pos, int total, int bi) {
  if (o->n_mirror >= o->num_layers) return KVC_OK;  // nothing is streamed
  // mirrored layers are [0, n_mirror): the next streamed one in this step, or the
  // first one of the next step
  const bool this_step = layer + 1 < o->num_layers;
  const int next = this_step ? std::max(layer + 1, o->n_mirror) : o->n_mirror;
  if (next == layer) return KVC_OK;
  for (const auto& B : o->b)
    if (B.layer == next) return KVC_OK;
  return start_fill(o, bi, next, this_step ? start_pos : total);
}

// Attend on a mirrored layer: bring the mirror up to rows [0, total) (in
// decode, just the appended row), then the resident path's kernels on the
// mirror's pages.  Same page geometry and split partition as the streamed path,
// so outputs are bit-identical.
int attend_mirrored(kvc_offload* o, const void* h_Q, void* h_Out, int layer, int q_len,
                    int start_pos, int num_heads, float scale, int causal, int total) {
  cudaStream_t s = o->compute;
  cudaError_t e;
  int rc;
  const int32_t* bt = static_cast<const int32_t*>(o->bt.ptr);
  constexpr int kChunkRows = 4096;
  int r0 = std::min(o->mirror_rows[layer], start_pos);  // the appended rows are new
  if (r0 < total) {
    const int chunk = std::min(kChunkRows, total - r0);
    const size_t cb = static_cast<size_t>(chunk) * o->row_bytes;
    if ((e = o->mstage_k.ensure(cb)) || (e = o->mstage_v.ensure(cb)))
      return cuda_error(e, "cudaMalloc(mirror staging)");
  }
  // Row chunks through the staging buffers on the compute stream (stream order
  // keeps a chunk's scatter ahead of the next chunk's copy into the staging).
  for (; r0 < total; r0 += kChunkRows) {
    const int n = std::min(kChunkRows, total - r0);
    const size_t off = static_cast<size_t>(layer) * o->layer_bytes +
                       static_cast<size_t>(r0) * o->row_bytes;
    const size_t nb = static_cast<size_t>(n) * o->row_bytes;
    if ((e = cudaMemcpyAsync(o->mstage_k.ptr, o->h_k + off, nb, cudaMemcpyHostToDevice, s)) ||
        (e = cudaMemcpyAsync(o->mstage_v.ptr, o->h_v + off, nb, cudaMemcpyHostToDevice, s)))
      return cuda_error(e, "cudaMemcpyAsync(mirror rows)");
    o->mirror_bytes += 2.0 * static_cast<double>(nb);
    if ((rc = do_append(&o->mirror, layer, o->mstage_k.ptr, o->mstage_v.ptr, bt, o->bt_len,
                        nullptr, nullptr, r0, n, s)))
      return rc;
  }
  o->mirror_rows[layer] = total;
  // the streamed layers keep coming in on the copy stream meanwhile
  if ((rc = prefetch_next(o, layer, start_pos, total, 1 - o->last_used))) return rc;

  const size_t qb = static_cast<size_t>(q_len) * num_heads * o->head_dim * o->es;
  if ((e = o->io.ensure(qb))) return cuda_error(e, "cudaMalloc(io)");
  uint8_t* d_q = static_cast<uint8_t*>(o->io.ptr);
  if ((rc = plan_queries(&o->plan, o->mirror.g, q_len, num_heads, start_pos, total, causal != 0,
                         o->device, s)))
    return rc;
  HostCallStage st;
  if ((rc = stage_q(o, h_Q, d_q, qb, h_Out, s, &st))) return rc;
  if ((rc = do_decode(&o->mirror, &o->plan, layer, d_q, st.out_dev, bt, o->bt_len, scale, s)))
    return rc;
  const PoolGeom& g = o->mirror.g;
  return finish_staged_call(s, h_Out, st, qb, "offload attend",
                            decode_uses_mma(g.dtype, g.head_dim, g.page_size));
}

}  // namespace

extern "C" int kvc_offload_create(void* h_k, void* h_v, int num_layers, int max_seq_len,
                                  int num_kv_heads, int head_dim, int dtype, int flags, int device,
                                  kvc_offload_t** out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  *out = nullptr;
  if (!h_k || !h_v) return set_error(KVC_ERR_INVALID_ARG, "host pools must not be null.");
  const int pages = max_seq_len > 0 ? (max_seq_len + kOffloadPageSize - 1) / kOffloadPageSize : 0;
  PoolGeom g;
  int rc = make_geom(1, std::max(1, pages), kOffloadPageSize, num_kv_heads, head_dim, dtype, &g);
  if (rc) return rc;
  if (num_layers <= 0 || max_seq_len <= 0)
    return set_error(KVC_ERR_INVALID_ARG, "KV cache dimensions must all be positive.");
  cudaError_t e;
  if (device < 0 && (e = cudaGetDevice(&device)) != cudaSuccess)
    return cuda_error(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_error(e, "cudaSetDevice");

  kvc_offload* o = new kvc_offload();
  o->device = device;
  o->num_layers = num_layers;
  o->max_seq_len = max_seq_len;
  o->num_kv_heads = num_kv_heads;
  o->head_dim = head_dim;
  o->dtype = dtype;
  o->es = g.elem_size;
  o->row_bytes = static_cast<size_t>(num_kv_heads) * head_dim * g.elem_size;
  o->layer_bytes = static_cast<size_t>(max_seq_len) * o->row_bytes;
  o->h_k = static_cast<uint8_t*>(h_k);
  o->h_v = static_cast<uint8_t*>(h_v);
  const size_t host_bytes = o->layer_bytes * num_layers;

  auto fail = [&](int code) {
    if (destroy_locked(o) == KVC_OK) delete o;  // nothing of it is queued yet
    return code;
  };
  if (flags & KVC_OFFLOAD_PINNED) {
    o->dma_ok = true;
  } else if (flags & KVC_OFFLOAD_REGISTER) {
    if (host_register(h_k, host_bytes) == cudaSuccess) {
      if (host_register(h_v, host_bytes) == cudaSuccess) {
        o->registered = true;
        o->dma_ok = true;
      } else {
        cudaHostUnregister(h_k);
      }
    }
    cudaGetLastError();  // a refused registration only means pageable copies
  }
  if ((e = cudaStreamCreateWithFlags(&o->copy, cudaStreamNonBlocking)) ||
      (e = cudaStreamCreateWithFlags(&o->compute, cudaStreamNonBlocking)))
    return fail(cuda_error(e, "cudaStreamCreate"));
  for (auto& B : o->b) {
    if ((e = B.k.ensure(o->layer_bytes)) || (e = B.v.ensure(o->layer_bytes)))
      return fail(cuda_error(e, "cudaMalloc(bounce)"));
    if ((e = cudaEventCreateWithFlags(&B.ready, cudaEventDisableTiming)) ||
        (e = cudaEventCreateWithFlags(&B.free, cudaEventDisableTiming)))
      return fail(cuda_error(e, "cudaEventCreate"));
    if ((e = cudaEventRecord(B.free, o->compute))) return fail(cuda_error(e, "cudaEventRecord"));
  }
  for (int i = 0; i < kTimingRing; ++i)
    if ((e = cudaEventCreate(&o->t_start[i])) || (e = cudaEventCreate(&o->t_stop[i])))
      return fail(cuda_error(e, "cudaEventCreate"));
  if ((rc = pool_alloc(&o->slot, g, device))) return fail(rc);
  if ((e = o->bt.ensure(sizeof(int32_t) * g.num_pages))) return fail(cuda_error(e, "cudaMalloc(bt)"));
  {
    std::vector<int32_t> ids(g.num_pages);
    for (int i = 0; i < g.num_pages; ++i) ids[i] = i;
    if ((e = cudaMemcpy(o->bt.ptr, ids.data(), sizeof(int32_t) * ids.size(), cudaMemcpyHostToDevice)))
      return fail(cuda_error(e, "cudaMemcpy(bt)"));
    o->bt_len = g.num_pages;
  }
  *out = o;
  return KVC_OK;
}

extern "C" int kvc_offload_destroy(kvc_offload_t* off) {
  if (!off) return KVC_OK;
  {
    std::lock_guard<std::mutex> lock(off->mu);
    if (const int rc = destroy_locked(off)) return rc;  // still in use: kept, call again
  }
  delete off;
  return KVC_OK;
}

extern "C" int kvc_offload_invalidate(kvc_offload_t* off) {
  if (!off) return set_error(KVC_ERR_INVALID_ARG, "offload handle must not be null.");
  std::lock_guard<std::mutex> lock(off->mu);
  for (auto& B : off->b) {
    B.layer = -1;
    B.rows = 0;
  }
  std::fill(off->mirror_rows.begin(), off->mirror_rows.end(), 0);
  return KVC_OK;
}

extern "C" int kvc_offload_set_mirror(kvc_offload_t* off, size_t budget_bytes, int* n_layers) {
  if (!off) return set_error(KVC_ERR_INVALID_ARG, "offload handle must not be null.");
  kvc_offload* o = off;
  std::lock_guard<std::mutex> lock(o->mu);
  cudaError_t e = cudaSetDevice(o->device);
  if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  if (const int rc = wait_stream(o->compute, "offload compute stream")) return rc;
  pool_release(&o->mirror);
  o->n_mirror = 0;
  o->mirror_rows.clear();
  const PoolGeom& sg = o->slot.g;
  const size_t per_layer = 2 * sg.layer_bytes;  // K and V pages of one layer
  const int n = static_cast<int>(std::min<size_t>(o->num_layers, budget_bytes / per_layer));
  if (n > 0) {
    PoolGeom g;
    int rc = make_geom(n, sg.num_pages, sg.page_size, sg.num_kv_heads, sg.head_dim, sg.dtype, &g);
    if (rc) return rc;
    if ((rc = pool_alloc(&o->mirror, g, o->device))) return rc;
    o->n_mirror = n;
    o->mirror_rows.assign(n, 0);
  }
  if (n_layers) *n_layers = o->n_mirror;
  return KVC_OK;
}

extern "C" int kvc_offload_mirror_stats(const kvc_offload_t* off, int* n_layers,
                                        double* uploaded_bytes) {
  if (!off) return set_error(KVC_ERR_INVALID_ARG, "offload handle must not be null.");
  kvc_offload* o = const_cast<kvc_offload*>(off);
  std::lock_guard<std::mutex> lock(o->mu);
  if (n_layers) *n_layers = o->n_mirror;
  if (uploaded_bytes) *uploaded_bytes = o->mirror_bytes;
  return KVC_OK;
}

extern "C" int kvc_offload_stats(const kvc_offload_t* off, double* h2d_bytes, double* h2d_ms,
                                 int64_t* prefetch_hits, int64_t* attend_calls) {
  if (!off) return set_error(KVC_ERR_INVALID_ARG, "offload handle must not be null.");
  kvc_offload* o = const_cast<kvc_offload*>(off);
  std::lock_guard<std::mutex> lock(o->mu);
  if (const int rc_dev = use_device(o->device)) return rc_dev;
  if (const int rc = harvest(o, true)) return rc;
  if (h2d_bytes) *h2d_bytes = o->h2d_bytes;
  if (h2d_ms) *h2d_ms = o->h2d_ms;
  if (prefetch_hits) *prefetch_hits = o->hits;
  if (attend_calls) *attend_calls = o->calls;
  return KVC_OK;
}

extern "C" int kvc_offload_attend(kvc_offload_t* off, const void* h_Q, const void* h_K_new,
                                  const void* h_V_new, void* h_Out, int layer_idx, int q_len,
                                  int start_pos, int num_heads, float scale, int causal) {
  if (!off) return set_error(KVC_ERR_INVALID_ARG, "offload handle must not be null.");
  kvc_offload* o = off;
  std::lock_guard<std::mutex> lock(o->mu);
  if (layer_idx < 0 || layer_idx >= o->num_layers)
    return set_error(KVC_ERR_OUT_OF_RANGE, "layer_idx out of range for the offloaded KV cache.");
  const int64_t total64 = static_cast<int64_t>(start_pos) + q_len;
  if (start_pos < 0 || q_len < 0 || total64 > o->max_seq_len)
    return set_error(KVC_ERR_OUT_OF_RANGE, "start_pos + q_len exceeds max_seq_len.");
  if (num_heads <= 0 || num_heads % o->num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be divisible by num_kv_heads.");
  if (q_len == 0) return KVC_OK;
  if (!h_Q || !h_Out || (!h_K_new) != (!h_V_new))
    return set_error(KVC_ERR_INVALID_ARG, "host buffers must not be null.");
  const int total = static_cast<int>(total64);
  cudaError_t e = cudaSetDevice(o->device);
  if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  o->calls++;
  harvest(o, false);  // never waits

  // 1. host append (kv_cache.py:222-225), unless the caller has written the rows
  //    already (null h_K_new / h_V_new).  A prefetch of this layer that covered
  //    rows >= start_pos is stale from start_pos on.
  if (h_K_new) {
    const size_t lay = static_cast<size_t>(layer_idx) * o->layer_bytes;
    const size_t off0 = static_cast<size_t>(start_pos) * o->row_bytes;
    const size_t nb = static_cast<size_t>(q_len) * o->row_bytes;
    memcpy(o->h_k + lay + off0, h_K_new, nb);
    memcpy(o->h_v + lay + off0, h_V_new, nb);
  }
  for (auto& B : o->b)
    if (B.layer == layer_idx && B.rows > start_pos) B.rows = start_pos;

  if (layer_idx < o->n_mirror) return attend_mirrored(o, h_Q, h_Out, layer_idx, q_len, start_pos,
                                                       num_heads, scale, causal, total);

  // 2. make rows [0, total) of the layer resident in a bounce buffer.
  int bi = -1;
  for (int i = 0; i < 2; ++i)
    if (o->b[i].layer == layer_idx) bi = i;
  int rc;
  if (bi >= 0) {
    o->hits++;
  } else {
    bi = 1 - o->last_used;
    if ((rc = start_fill(o, bi, layer_idx, 0))) return rc;
  }
  kvc_offload::Bounce& B = o->b[bi];
  if ((rc = copy_rows(o, bi, layer_idx, B.rows, total))) return rc;
  B.rows = total;
  if ((e = cudaEventRecord(B.ready, o->copy))) return cuda_error(e, "cudaEventRecord(ready)");
  o->last_used = bi;

  // 3. prefetch the next streamed layer into the other bounce buffer.
  if ((rc = prefetch_next(o, layer_idx, start_pos, total, 1 - bi))) return rc;

  // 4. compute stream: scatter the rows into the paged slot, attend, copy out.
  const size_t qb = static_cast<size_t>(q_len) * num_heads * o->head_dim * o->es;
  if ((e = o->io.ensure(qb))) return cuda_error(e, "cudaMalloc(io)");
  uint8_t* d_q = static_cast<uint8_t*>(o->io.ptr);
  cudaStream_t s = o->compute;
  HostCallStage st;
  if ((rc = stage_q(o, h_Q, d_q, qb, h_Out, s, &st))) return rc;
  if ((e = cudaStreamWaitEvent(s, B.ready, 0))) return cuda_error(e, "cudaStreamWaitEvent");
  const int32_t* bt = static_cast<const int32_t*>(o->bt.ptr);
  if ((rc = do_append(&o->slot, 0, B.k.ptr, B.v.ptr, bt, o->bt_len, nullptr, nullptr, 0, total, s)))
    return rc;
  if ((e = cudaEventRecord(B.free, s))) return cuda_error(e, "cudaEventRecord(free)");
  if ((rc = plan_queries(&o->plan, o->slot.g, q_len, num_heads, start_pos, total, causal != 0,
                         o->device, s)))
    return rc;
  if ((rc = do_decode(&o->slot, &o->plan, 0, d_q, st.out_dev, bt, o->bt_len, scale, s))) return rc;
  const PoolGeom& g = o->slot.g;
  return finish_staged_call(s, h_Out, st, qb, "offload attend",
                            decode_uses_mma(g.dtype, g.head_dim, g.page_size));
}
