// Head exchange: KV heads split across the GPUs of one node, per-head outputs
// pushed to every rank by the merge kernel itself.
//
// The reference runs one model on one GPU and has no multi-device path.  When
// the KV heads of a layer are split over N GPUs (one process each), every rank
// needs all heads of the attention output before the next layer's output
// projection.  Instead of a separate all-gather after the decode, the merge
// kernel stores each finished output row into the exchange slot of every rank
// over NVLink (plain peer stores; the peers' buffers are mapped with CUDA IPC);
// a one-warp kernel behind it then publishes a per-step epoch in a flag word on
// every rank and waits, with a time limit, until all ranks have published it.
// Nothing crosses NVLink but the outputs and the flags.
#include <cuda_runtime.h>

#include <cstring>

#include "kvcache.h"
#include "kvc_common.h"

using namespace kvc;

static_assert(sizeof(cudaIpcMemHandle_t) <= KVC_XCHG_HANDLE_BYTES, "IPC handle size");

namespace {

void unmap_peers(kvc_xchg* x) {
  for (int p = 0; p < kMaxPeers; ++p) {
    if (x->ipc_opened[p] && x->peer_base[p]) cudaIpcCloseMemHandle(x->peer_base[p]);
    x->ipc_opened[p] = false;
    x->peer_base[p] = nullptr;
  }
  x->connected = false;
}

}  // namespace

extern "C" int kvc_xchg_create(int device, int rank, int world, size_t slot_bytes, int n_slots,
                               kvc_xchg_t** out) {
  if (!out) return set_error(KVC_ERR_INVALID_ARG, "out must not be null.");
  *out = nullptr;
  if (world < 1 || world > kMaxPeers)
    return set_error(KVC_ERR_INVALID_ARG, "world must be in [1, %d].", kMaxPeers);
  if (rank < 0 || rank >= world) return set_error(KVC_ERR_INVALID_ARG, "rank must be in [0, world).");
  if (slot_bytes == 0 || n_slots <= 0)
    return set_error(KVC_ERR_INVALID_ARG, "slot_bytes and n_slots must be positive.");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  auto* x = new kvc_xchg();
  x->device = device;
  x->rank = rank;
  x->world = world;
  x->slot_bytes = slot_bytes;
  x->slot_stride = (slot_bytes + 255) & ~static_cast<size_t>(255);
  x->n_slots = n_slots;
  const size_t bytes = kXchgSlotsOff + x->slot_stride * static_cast<size_t>(n_slots);
  if ((e = dev_alloc(reinterpret_cast<void**>(&x->base), bytes)) != cudaSuccess) {
    delete x;
    return cuda_error(e, "cudaMalloc(exchange buffer)");
  }
  // flags (epoch 0 = nothing published yet) and the completion counter start at zero
  if ((e = cudaMemset(x->base, 0, kXchgSlotsOff)) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(x->base);
    delete x;
    return cuda_error(e, "cudaMemset(exchange flags)");
  }
  *out = x;
  return KVC_OK;
}

extern "C" int kvc_xchg_handle(const kvc_xchg_t* x, void* handle_out) {
  if (!x || !handle_out) return set_error(KVC_ERR_INVALID_ARG, "exchange and handle_out must not be null.");
  if (const int rc_dev = use_device(x->device)) return rc_dev;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, x->base);
  if (e != cudaSuccess) return cuda_error(e, "cudaIpcGetMemHandle");
  memset(handle_out, 0, KVC_XCHG_HANDLE_BYTES);
  memcpy(handle_out, &h, sizeof(h));
  return KVC_OK;
}

extern "C" int kvc_xchg_connect(kvc_xchg_t* x, const void* handles) {
  if (!x || !handles) return set_error(KVC_ERR_INVALID_ARG, "exchange and handles must not be null.");
  cudaError_t e = cudaSetDevice(x->device);
  if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
  unmap_peers(x);
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int p = 0; p < x->world; ++p) {
    if (p == x->rank) {
      x->peer_base[p] = x->base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + static_cast<size_t>(p) * KVC_XCHG_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    if ((e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
      unmap_peers(x);
      return cuda_error(e, "cudaIpcOpenMemHandle");
    }
    x->peer_base[p] = static_cast<uint8_t*>(ptr);
    x->ipc_opened[p] = true;
  }
  x->connected = true;
  return KVC_OK;
}

extern "C" int kvc_xchg_connect_ptrs(kvc_xchg_t* x, void* const* peer_bases) {
  if (!x || !peer_bases) return set_error(KVC_ERR_INVALID_ARG, "exchange and peer_bases must not be null.");
  unmap_peers(x);
  for (int p = 0; p < x->world; ++p) {
    if (!peer_bases[p] || (reinterpret_cast<uintptr_t>(peer_bases[p]) & 255u)) {
      unmap_peers(x);
      return set_error(KVC_ERR_INVALID_ARG, "peer buffer %d is null or not 256-byte aligned.", p);
    }
    x->peer_base[p] = static_cast<uint8_t*>(peer_bases[p]);
  }
  if (x->peer_base[x->rank] != x->base) {
    unmap_peers(x);
    return set_error(KVC_ERR_INVALID_ARG, "peer_bases[rank] must be this rank's own buffer.");
  }
  x->connected = true;
  return KVC_OK;
}

extern "C" int kvc_xchg_base(const kvc_xchg_t* x, void** d_base) {
  if (!x || !d_base) return set_error(KVC_ERR_INVALID_ARG, "exchange and d_base must not be null.");
  *d_base = x->base;
  return KVC_OK;
}

extern "C" int kvc_xchg_slot(const kvc_xchg_t* x, int slot, void** d_ptr) {
  if (!x || !d_ptr) return set_error(KVC_ERR_INVALID_ARG, "exchange and d_ptr must not be null.");
  if (slot < 0 || slot >= x->n_slots) return set_error(KVC_ERR_OUT_OF_RANGE, "slot out of range.");
  *d_ptr = x->base + kXchgSlotsOff + static_cast<size_t>(slot) * x->slot_stride;
  return KVC_OK;
}

extern "C" int kvc_xchg_set_wait_limit(kvc_xchg_t* x, double seconds) {
  if (!x) return set_error(KVC_ERR_INVALID_ARG, "exchange must not be null.");
  if (!(seconds > 0.0) || seconds > 60.0)
    return set_error(KVC_ERR_INVALID_ARG, "wait limit must be in (0, 60] seconds.");
  x->wait_limit_ns = static_cast<unsigned long long>(seconds * 1e9);
  return KVC_OK;
}

extern "C" int kvc_xchg_destroy(kvc_xchg_t* x) {
  if (!x) return KVC_OK;
  cudaSetDevice(x->device);
  cudaDeviceSynchronize();
  unmap_peers(x);
  if (x->base) cudaFree(x->base);
  delete x;
  return KVC_OK;
}

extern "C" int kvc_append_decode_xchg(kvc_pool_t* pool, const kvc_plan_t* plan, int layer,
                                      const void* d_q, const void* d_k_new, const void* d_v_new,
                                      kvc_xchg_t* x, int slot, int total_heads, int head_offset,
                                      const int32_t* d_block_tables, int bt_stride, float scale,
                                      void* stream) {
  if (!pool || !plan || !x) return set_error(KVC_ERR_INVALID_ARG, "pool, plan and exchange must not be null.");
  if (!plan->valid) return set_error(KVC_ERR_INVALID_ARG, "plan has not been built.");
  if (!x->connected) return set_error(KVC_ERR_INVALID_ARG, "exchange is not connected to its peers.");
  if (x->device != pool->device)
    return set_error(KVC_ERR_INVALID_ARG, "exchange and pool live on different devices.");
  if (slot < 0 || slot >= x->n_slots) return set_error(KVC_ERR_OUT_OF_RANGE, "slot out of range.");
  if (head_offset < 0 || plan->num_heads <= 0 || head_offset + plan->num_heads > total_heads)
    return set_error(KVC_ERR_INVALID_ARG, "heads [%d, %d) do not fit in %d heads.", head_offset,
                     head_offset + plan->num_heads, total_heads);
  const size_t need = static_cast<size_t>(plan->n_queries) * total_heads * pool->g.head_dim *
                      pool->g.elem_size;
  if (need > x->slot_bytes)
    return set_error(KVC_ERR_INVALID_ARG, "a slot holds %zu bytes, the outputs need %zu.",
                     x->slot_bytes, need);
  if (const int rc_dev = use_device(pool->device)) return rc_dev;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XchgTarget xt{x, slot, total_heads, head_offset};
  if (!d_k_new && !d_v_new)
    return do_decode_fused(pool, plan, layer, d_q, nullptr, d_block_tables, bt_stride, scale,
                           nullptr, nullptr, s, &xt);
  return append_then_decode(pool, plan, layer, d_q, d_k_new, d_v_new, nullptr, d_block_tables,
                            bt_stride, scale, s, &xt);
}
