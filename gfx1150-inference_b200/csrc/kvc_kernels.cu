// CUDA kernels of the B200 KV-cache decode path (sm_100a):
//   append_kernel             fused, vectorised scatter of new K/V rows into the paged pool
//   decode_persistent_kernel  split-K flash-decoding GQA attention, 16-bit storage: one
//                             CTA per SM, warps streaming KV slabs through bulk-copy rings,
//                             tensor-core math, the row append fused in
//   merge_splits_kernel       merge of the split partials (programmatic dependent launch);
//                             with KV heads split over GPUs it stores the rows into every
//                             rank's exchange slot
//   xchg_signal_kernel        publishes the head exchange's epoch and waits for the peers
//   decode_simt_kernel        split-K GQA attention on CUDA cores (fp32 storage, other
//                             head dims), splits merged by the last CTA of a query
//   stage_inputs_kernel       page-locked host inputs -> device staging (host-buffer calls)
//   rope_kernel               rotary position embedding (rope.hip semantics)
//   gather_kernel             pool -> token-major rows (bit-exact pool checks)
//   fill_normal_kernel        seeded N(0, s^2) synthetic pool contents
//
// The attention computes, for every query m and q-head h, exactly the quantity of
// gfx1150-inference's gqa_online_softmax_kernel (src/kernels/attention.hip:35-123):
//   kv_h = h / (H / Hkv)                                   (attention.hip:59-60)
//   score_j = (q . k_j) * scale, scale used as given        (attention.hip:99)
//   out = sum_j softmax(score)_j * v_j over j < ctx        (attention.hip:75-113)
//   out = 0 when nothing is attended                       (attention.hip:115)
// with fp32 accumulation.  The work is organised the B200 way instead of one
// wave per (m, h) scanning every position: a query's context is cut into splits
// of fixed length; each split of one KV head is streamed from HBM once, 16
// positions at a time through shared memory, and serves all q-heads of the
// group from the same tile; the splits' partial softmax states are then merged.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "kvc_common.h"
#include "kvc_device.cuh"
#include "kvc_internal.h"
#include "kvcache.h"

namespace kvc {

// ---- device error word -----------------------------------------------------------
// [0] = first error code (KVC_DEVERR_*), [1] = auxiliary value.  One copy per
// device; read by the host after synchronising.
__device__ uint32_t g_kvc_deverr[2];

__device__ __forceinline__ void report_error(uint32_t code, uint32_t info) {
  if (atomicCAS(&g_kvc_deverr[0], 0u, code) == 0u) g_kvc_deverr[1] = info;
}

cudaError_t device_error_address(void** p) { return cudaGetSymbolAddress(p, g_kvc_deverr); }

cudaError_t read_device_error(uint32_t* code, uint32_t* info, bool clear) {
  uint32_t w[2] = {0, 0};
  cudaError_t e = cudaMemcpyFromSymbol(w, g_kvc_deverr, sizeof(w));
  if (e != cudaSuccess) return e;
  if (code) *code = w[0];
  if (info) *info = w[1];
  if (clear && (w[0] | w[1])) {
    const uint32_t z[2] = {0, 0};
    e = cudaMemcpyToSymbol(g_kvc_deverr, z, sizeof(z));
  }
  return e;
}

// =====================================================================================
// Append: one thread moves one 16-byte unit of K and the same unit of V.
// Replaces the two blocking row copies of the reference (attention.hip:336-341
// host->device, :410-415 device->device) with one coalesced scatter for all rows.
// =====================================================================================
__global__ void __launch_bounds__(256) append_kernel(const AppendArgs a) {
  const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t per_row = static_cast<size_t>(a.num_kv_heads) * a.row_units;
  if (idx >= per_row * a.n) return;
  const int i = static_cast<int>(idx / per_row);
  const int rem = static_cast<int>(idx - static_cast<size_t>(i) * per_row);
  const int h = rem / a.row_units;
  const int u = rem - h * a.row_units;

  const int pos = a.positions ? a.positions[i] : a.pos0 + i;
  const int row = a.rows ? a.rows[i] : 0;
  const int slot = pos / a.page_size;
  if (pos < 0 || slot >= a.bt_stride) {
    report_error(3u /*KVC_DEVERR_BAD_POSITION*/, static_cast<uint32_t>(pos));
    return;
  }
  const int phys = a.block_tables[static_cast<size_t>(row) * a.bt_stride + slot];
  if (phys < 0 || phys >= a.num_pages) {
    report_error(1u /*KVC_DEVERR_BAD_PAGE*/, static_cast<uint32_t>(phys));
    return;
  }
  const int t = pos - slot * a.page_size;
  const size_t dst = (static_cast<size_t>(phys) * a.num_kv_heads + h) * a.page_head_bytes +
                     unit_offset(a.layout, t, u, a.row_units) * 16;
  const size_t src = (static_cast<size_t>(i) * a.num_kv_heads + h) * a.row_units * 16 +
                     static_cast<size_t>(u) * 16;
  const uint4 kv = *reinterpret_cast<const uint4*>(a.k_new + src);
  const uint4 vv = *reinterpret_cast<const uint4*>(a.v_new + src);
  *reinterpret_cast<uint4*>(a.k_layer + dst) = kv;
  *reinterpret_cast<uint4*>(a.v_layer + dst) = vv;
}

cudaError_t launch_append(const AppendArgs& a, int /*elem_size*/, cudaStream_t s) {
  const size_t total = static_cast<size_t>(a.n) * a.num_kv_heads * a.row_units;
  if (total == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  append_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

// =====================================================================================
// Gather: pool -> (count, Hkv, D) rows of one sequence.
// =====================================================================================
__global__ void __launch_bounds__(256) gather_kernel(const GatherArgs a) {
  const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t per_row = static_cast<size_t>(a.num_kv_heads) * a.row_units;
  if (idx >= per_row * a.count) return;
  const int i = static_cast<int>(idx / per_row);
  const int rem = static_cast<int>(idx - static_cast<size_t>(i) * per_row);
  const int h = rem / a.row_units;
  const int u = rem - h * a.row_units;
  const int pos = a.start + i;
  const int slot = pos / a.page_size;
  const int phys = (slot < a.bt_stride) ? a.bt_row[slot] : -1;
  const size_t dst = (static_cast<size_t>(i) * a.num_kv_heads + h) * a.row_units * 16 +
                     static_cast<size_t>(u) * 16;
  if (phys < 0 || phys >= a.num_pages) {
    report_error(1u, static_cast<uint32_t>(phys));
    *reinterpret_cast<uint4*>(a.k_out + dst) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(a.v_out + dst) = make_uint4(0, 0, 0, 0);
    return;
  }
  const int t = pos - slot * a.page_size;
  const size_t src = (static_cast<size_t>(phys) * a.num_kv_heads + h) * a.page_head_bytes +
                     unit_offset(a.layout, t, u, a.row_units) * 16;
  *reinterpret_cast<uint4*>(a.k_out + dst) = *reinterpret_cast<const uint4*>(a.k_layer + src);
  *reinterpret_cast<uint4*>(a.v_out + dst) = *reinterpret_cast<const uint4*>(a.v_layer + src);
}

cudaError_t launch_gather(const GatherArgs& a, cudaStream_t s) {
  const size_t total = static_cast<size_t>(a.count) * a.num_kv_heads * a.row_units;
  if (total == 0) return cudaSuccess;
  gather_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(a);
  return cudaGetLastError();
}

// =====================================================================================
// Input staging for the host-buffer entry points: q and the new K/V rows are read
// straight from page-locked host memory (over PCIe) into device staging.  The
// kernel triggers its dependents first, so the decode launched behind it streams
// KV from HBM while the inputs cross the host link; the decode reads them only
// after griddepcontrol.wait.  Its CTAs are small enough to share an SM with a
// decode CTA (4 warps at <= 32 registers: the 4,096 registers a 240-register
// decode CTA leaves free, and no shared memory), so the decode's CTAs start on
// every SM at once instead of waiting for the SMs the staging holds.
// =====================================================================================
constexpr int kStageThreads = 128;
constexpr int kStageUnroll = 4;  // 16-byte loads in flight per thread

__global__ void __launch_bounds__(kStageThreads, 16) stage_inputs_kernel(const StageArgs a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const unsigned stride = gridDim.x * blockDim.x;
  const unsigned t0 = blockIdx.x * blockDim.x + threadIdx.x;
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    // staging sizes are far below 2^32 16-byte units (checked by the launcher)
    const unsigned n16 = static_cast<unsigned>(a.bytes[b] / 16);
    const uint4* src = reinterpret_cast<const uint4*>(a.src[b]);
    uint4* dst = reinterpret_cast<uint4*>(a.dst[b]);
#pragma unroll 1
    for (unsigned i0 = t0; i0 < n16; i0 += kStageUnroll * stride) {
      uint4 v[kStageUnroll];
#pragma unroll
      for (int u = 0; u < kStageUnroll; ++u)
        if (i0 + u * stride < n16) v[u] = src[i0 + u * stride];
#pragma unroll
      for (int u = 0; u < kStageUnroll; ++u)
        if (i0 + u * stride < n16) dst[i0 + u * stride] = v[u];
    }
    for (size_t i = static_cast<size_t>(n16) * 16 + t0; i < a.bytes[b]; i += stride)
      a.dst[b][i] = a.src[b][i];
  }
}

cudaError_t launch_stage_inputs(const StageArgs& a, cudaStream_t s) {
  // Same shared-memory carveout as the decode kernel, so a staging CTA never
  // keeps an SM in a configuration a decode CTA cannot join.
  static std::atomic<bool> carveout_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  if (dev >= 0 && dev < 64 && !carveout_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(stage_inputs_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) == cudaSuccess)
      carveout_set[dev].store(true, std::memory_order_release);
    else
      cudaGetLastError();  // a preference only: the staging still runs
  }
  const size_t n16 = (a.bytes[0] + a.bytes[1] + a.bytes[2]) / 16 + 1;
  if (n16 >= (static_cast<size_t>(1) << 31)) return cudaErrorInvalidValue;
  const size_t per_cta = static_cast<size_t>(kStageThreads) * kStageUnroll;
  const unsigned grid = static_cast<unsigned>(std::min<size_t>(64, (n16 + per_cta - 1) / per_cta));
  stage_inputs_kernel<<<grid, kStageThreads, 0, s>>>(a);
  return cudaGetLastError();
}

// =====================================================================================
// Rotary position embedding (rope.hip:21-55 semantics): one thread per rotation
// pair.  As the staging step of the rotate + append + attend path it triggers its
// dependents first, so the decode behind it streams KV while q and the new K rows
// are rotated; the decode reads them only after griddepcontrol.wait.
// =====================================================================================
template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const RopeArgs a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int half = a.head_dim / 2;
  const size_t n0 = static_cast<size_t>(a.n_tokens) * a.heads[0] * half;
  const size_t n1 = static_cast<size_t>(a.n_tokens) * a.heads[1] * half;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < n0 + n1;
       idx += stride) {
    const int b = idx < n0 ? 0 : 1;
    const size_t r = b == 0 ? idx : idx - n0;
    const int i = static_cast<int>(r % half);
    const size_t th = r / half;                       // token * heads + head
    const int t = static_cast<int>(th / a.heads[b]);
    const int pos = a.positions ? a.positions[t] : a.pos0 + t;
    const float angle = static_cast<float>(pos) * a.inv_freq[i];
    float sn, cs;
    sincosf(angle, &sn, &cs);
    const int i0 = a.neox ? i : 2 * i;
    const int i1 = a.neox ? i + half : 2 * i + 1;
    const T* x = reinterpret_cast<const T*>(a.src[b]) + th * a.head_dim;
    T* y = reinterpret_cast<T*>(a.dst[b]) + th * a.head_dim;
    const float v0 = to_f32<T>(x[i0]), v1 = to_f32<T>(x[i1]);
    y[i0] = from_f32<T>(v0 * cs - v1 * sn);
    y[i1] = from_f32<T>(v0 * sn + v1 * cs);
  }
}

cudaError_t launch_rope(const RopeArgs& a, cudaStream_t s, bool pdl) {
  const size_t pairs =
      static_cast<size_t>(a.n_tokens) * (a.heads[0] + a.heads[1]) * (a.head_dim / 2);
  if (pairs == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<size_t>(148 * 8, (pairs + 255) / 256)), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (a.dtype) {
    case 0: return cudaLaunchKernelEx(&cfg, rope_kernel<__half>, a);
    case 1: return cudaLaunchKernelEx(&cfg, rope_kernel<__nv_bfloat16>, a);
    case 2: return cudaLaunchKernelEx(&cfg, rope_kernel<float>, a);
    default: return cudaErrorInvalidValue;
  }
}

// =====================================================================================
// Seeded normal fill (synthetic benchmark contents).  Counter-based: element i
// of the pool always receives the same value for a given seed.
// =====================================================================================
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256) fill_normal_kernel(const FillArgs a) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n_elems;
       i += stride) {
    const uint64_t r = mix64(a.seed ^ mix64(a.index0 + i));
    // Box-Muller on two 24-bit uniforms in (0, 1].
    const float u1 = (static_cast<float>(r >> 40) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((r >> 8) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2) * a.stddev;
    if (a.dtype == 2) {
      reinterpret_cast<float*>(a.base)[i] = z;
    } else if (a.dtype == 1) {
      reinterpret_cast<__nv_bfloat16*>(a.base)[i] = __float2bfloat16_rn(z);
    } else {
      reinterpret_cast<__half*>(a.base)[i] = __float2half_rn(z);
    }
  }
}

cudaError_t launch_fill_normal(const FillArgs& a, cudaStream_t s) {
  if (a.n_elems == 0) return cudaSuccess;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  const int sms = device_sms(dev);
  const size_t want = (a.n_elems + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(want < static_cast<size_t>(sms) * 16 ? want : sms * 16);
  fill_normal_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

// =====================================================================================
// Split merge, shared by both attention kernels.
//
// Every CTA of a query with n_splits > 1 leaves (M, L, O) for its q-heads in the
// partial buffers, O unnormalised relative to the running max M (log2 units).
// The last CTA to finish combines them in split order:
//   M* = max_k M_k,  L* = sum_k L_k 2^(M_k - M*),  out = sum_k O_k 2^(M_k - M*) / L*
// Shared memory: wt[8][kMergeChunk] weights + acc[8][D] + stats[16].
// =====================================================================================
constexpr int kMergeChunk = 128;
// Bytes reserved at the start of dynamic shared memory for the mbarriers.
constexpr int kBarBytes = 256;

__device__ __forceinline__ size_t merge_smem_bytes(int head_dim) {
  return (8 * kMergeChunk + 8 * static_cast<size_t>(head_dim) + 16) * sizeof(float);
}

template <typename T>
__device__ void merge_splits(const DecodeArgs& a, float* sm, int query, int split_base,
                             int n_splits, int hq0, int nh) {
  const int D = a.head_dim;
  const int H = a.num_heads;
  float* wt = sm;                        // [8][kMergeChunk]
  float* acc = wt + 8 * kMergeChunk;     // [8][D]
  float* st = acc + 8 * D;               // [8] max, [8] 1/sum
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;

  // 1. per-head max and sum (one warp per head, lanes stride over splits, then a
  //    fixed-order butterfly: the result does not depend on which CTA merges).
  for (int h = warp; h < nh; h += nwarps) {
    float mx = kNegBig;
    for (int k = lane; k < n_splits; k += 32)
      mx = fmaxf(mx, __ldcg(&a.part_ml[static_cast<size_t>(split_base + k) * H + hq0 + h]).x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int k = lane; k < n_splits; k += 32) {
      const float2 ml = __ldcg(&a.part_ml[static_cast<size_t>(split_base + k) * H + hq0 + h]);
      sum += ml.y * fast_exp2(ml.x - mx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      st[h] = mx;
      st[8 + h] = sum > 0.f ? 1.0f / sum : 0.f;
    }
  }
  for (int i = threadIdx.x; i < nh * D; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();

  // 2. weighted sum of the partial outputs, chunk by chunk of splits.
  for (int k0 = 0; k0 < n_splits; k0 += kMergeChunk) {
    const int kn = min(kMergeChunk, n_splits - k0);
    for (int i = threadIdx.x; i < nh * kn; i += blockDim.x) {
      const int h = i / kn, k = i - (i / kn) * kn;
      const float m = __ldcg(&a.part_ml[static_cast<size_t>(split_base + k0 + k) * H + hq0 + h]).x;
      wt[h * kMergeChunk + k] = fast_exp2(m - st[h]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
      const int h = i / D, d = i - (i / D) * D;
      float o = acc[i];
      const float* src = a.part_o + (static_cast<size_t>(split_base + k0) * H + hq0 + h) * D + d;
      for (int k = 0; k < kn; ++k)
        o += __ldcg(src + static_cast<size_t>(k) * H * D) * wt[h * kMergeChunk + k];
      acc[i] = o;
    }
    __syncthreads();
  }
  T* out = reinterpret_cast<T*>(a.out) + (static_cast<size_t>(query) * H + hq0) * D;
  for (int i = threadIdx.x; i < nh * D; i += blockDim.x) out[i] = from_f32<T>(acc[i] * st[8 + i / D]);
}

// Fused append, global half: lanes of one warp copy query `query`'s new K and V
// row of head `kvh` into the pool at position pos (16-byte units).
__device__ __forceinline__ void append_row_to_pool(const DecodeArgs& a, int layout, int es,
                                                   int query, int kvh, int pos,
                                                   const int32_t* bt_row, int lane) {
  const int U = a.head_dim * es / 16;
  const int slot = pos / a.page_size;
  const int phys = slot < a.bt_stride ? bt_row[slot] : -1;
  if (phys < 0 || phys >= a.num_pages) return;  // reported by the slab loader
  const int t = pos - slot * a.page_size;
  const size_t page_head = static_cast<size_t>(a.page_size) * a.head_dim * es;
  const size_t dst = (static_cast<size_t>(phys) * a.num_kv_heads + kvh) * page_head;
  const size_t src = (static_cast<size_t>(query) * a.num_kv_heads + kvh) * U * 16;
  uint8_t* kl = const_cast<uint8_t*>(a.k_layer);
  uint8_t* vl = const_cast<uint8_t*>(a.v_layer);
  for (int x = lane; x < 2 * U; x += 32) {
    const int u = x % U;
    const uint8_t* sp = (x < U ? a.k_new : a.v_new) + src + static_cast<size_t>(u) * 16;
    uint8_t* dp = (x < U ? kl : vl) + dst + unit_offset(layout, t, u, U) * 16;
    *reinterpret_cast<uint4*>(dp) = *reinterpret_cast<const uint4*>(sp);
  }
}

// Fused append, shared half: overwrite row t of a staged K/V slab pair with the
// new row (the bulk copy may have fetched the pool's previous contents).
__device__ __forceinline__ void patch_slab_row(const DecodeArgs& a, int layout, int es, uint8_t* st,
                                               int slab_bytes, int query, int kvh, int t, int tid,
                                               int nthreads) {
  const int U = a.head_dim * es / 16;
  const size_t src = (static_cast<size_t>(query) * a.num_kv_heads + kvh) * U * 16;
  for (int x = tid; x < 2 * U; x += nthreads) {
    const int u = x % U;
    const uint8_t* sp = (x < U ? a.k_new : a.v_new) + src + static_cast<size_t>(u) * 16;
    *reinterpret_cast<uint4*>(st + (x < U ? 0 : slab_bytes) + unit_offset(layout, t, u, U) * 16) =
        *reinterpret_cast<const uint4*>(sp);
  }
}

// Publish this CTA's partial and let the last CTA of (query, KV head, head chunk)
// merge.  Classic threadfence reduction: no CTA ever waits for another.
template <typename T>
__device__ void finish_split(const DecodeArgs& a, float* sm, int query, int kvh, int hc,
                             int split_base, int n_splits, int hq0, int nh) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const size_t cidx = (static_cast<size_t>(query) * a.num_kv_heads + kvh) * a.n_hchunk + hc;
    const unsigned prev = atomicAdd(&a.counters[cidx], 1u);
    s_last = (prev == static_cast<unsigned>(n_splits) - 1u);
    if (s_last) a.counters[cidx] = 0u;  // every other split has arrived: re-arm
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  merge_splits<T>(a, sm, query, split_base, n_splits, hq0, nh);
}

// =====================================================================================
// Persistent tensor-core decode kernel (16-bit storage, head_dim multiple of 32).
//
// kPersistCtasPerSm CTAs of NW warps per SM; every warp is an independent
// streaming engine.
// The host lists whole split units (one split of one query for one KV head and
// <= 8 of its q-heads) longest first; warp w of the grid starts with unit w and
// then takes the next unlisted unit from a global counter, so every warp keeps
// streaming until the list is done.  A warp's producer side keeps NS slabs (16
// positions of K and V, one bulk copy each) in flight in the warp's
// shared-memory ring, running into the next unit before the current one is
// finished, and fetches the next unit's record and page ids one step per
// issued slab; its consumer side does the math of a slab
// as soon as it lands (S = Q K^T, online softmax, O^T += V^T P^T, mma.sync
// m16n8k16) and, at the end of a unit, writes the output or the split's
// partial state (merged by merge_splits_kernel, launched behind it).
// There is no CTA-wide synchronisation after start-up.
// =====================================================================================
constexpr int kPersistBarBytes = 512;    // NW * NS mbarriers
constexpr int kPersistMetaBytes = 4096;  // NW * NS stage records (4 x int4 each)

template <int D>
constexpr int persist_stages() {
  // ~192 KiB of ring per SM (24 KiB per warp), at most 12 stages per warp
  return (196608 / (kPersistWarpsPerSm * 2 * kSlab * D * 2)) > 12
             ? 12
             : (196608 / (kPersistWarpsPerSm * 2 * kSlab * D * 2));
}

template <typename T, int D, int NW, int NS>
__global__ void __launch_bounds__(NW * 32, kPersistCtasPerSm)
    decode_persistent_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int SLAB_BYTES = kSlab * D * 2;
  constexpr int STAGE_BYTES = 2 * SLAB_BYTES;
  constexpr int KC = D / 16;
  constexpr int MT = D / 16;
  constexpr int U = D / 8;
  static_assert(NW * NS * 8 <= kPersistBarBytes, "mbarrier block too small");
  static_assert(NW * NS * 64 <= kPersistMetaBytes, "stage record block too small");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int ps = a.page_size;
  const int spp = ps / kSlab;  // slabs per page
  const int H = a.num_heads;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * NS;
  int4* meta = reinterpret_cast<int4*>(smem + kPersistBarBytes) + warp * NS * 4;
  uint8_t* stages = smem + kPersistBarBytes + kPersistMetaBytes + warp * NS * STAGE_BYTES;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int gw = blockIdx.x * NW + warp;
  const int W = gridDim.x * NW;
  // A graph-stable plan keeps its counts in the plan's device header (its launches
  // are replayed as contexts grow); otherwise they come with the launch.
  const int n_units = a.plan_hdr ? a.plan_hdr[kHdrUnits] : a.n_units;
  const int l2_ahead = a.plan_hdr ? a.plan_hdr[kHdrL2Ahead] : a.l2_ahead;
  const size_t page_stride = static_cast<size_t>(a.num_kv_heads) * ps * D * 2;
  const uint64_t policy = l2_policy_evict_first();

  // Unit record r (3 x int4): {query, split, tb, te}, {bt row, ctx, slot0, n_splits},
  // {kvh, hc, hq0, nh}.
  auto load_pages = [&](const int4& r0, const int4& r1, int& pg0, int& page0, int& page1) {
    pg0 = r0.z / ps;
    const int npages = (r0.w + ps - 1) / ps - pg0;
    const int32_t* bt_row = a.block_tables + static_cast<size_t>(r1.x) * a.bt_stride;
    page0 = page1 = -1;
    // A replayed launch of a rebuilt plan skips the host's check of the contexts
    // against the table width: an entry past the row's end counts as a bad page.
    if (lane < npages) {
      const int v = pg0 + lane < a.bt_stride ? bt_row[pg0 + lane] : -1;
      page0 = (v >= 0 && v < a.num_pages) ? v : -1;
      if (page0 < 0) report_error(1u, static_cast<uint32_t>(v));
    }
    if (lane + 32 < npages) {
      const int v = pg0 + lane + 32 < a.bt_stride ? bt_row[pg0 + lane + 32] : -1;
      page1 = (v >= 0 && v < a.num_pages) ? v : -1;
      if (page1 < 0) report_error(1u, static_cast<uint32_t>(v));
    }
  };

  // ---------------- producer ----------------
  // Units are stored longest first.  Warp gw starts with unit gw and then takes
  // the next free one from a global counter (dynamic list scheduling, so every
  // SM keeps streaming until the whole list is done).  p_*: the unit being
  // issued.  n_*: the next unit, fetched while the current one streams, one
  // step per issued slab (counter ticket, then its record, then its page ids),
  // so unit switches never wait on memory.  pq: Q fragments of the unit the
  // producer started last, taken over by the consumer when it reaches it.
  int p_pos = gw;
  int4 p_r0 = make_int4(0, 0, 0, 0), p_r1 = p_r0, p_r2 = p_r0;
  int p_j = 0, p_end = 0, p_pg0 = 0, p_page0 = -1, p_page1 = -1;
  int4 n_r0 = p_r0, n_r1 = p_r0, n_r2 = p_r0;
  int n_pg0 = 0, n_page0 = -1, n_page1 = -1;
  int n_state = 0;  // 0: nothing, 1: ticket taken, 2: record fetched, 3: page ids fetched, 4: none left
  int n_pos = -1;
  unsigned n_ticket = 0;
  constexpr bool kPrefetchQ = D <= 128;  // registers allow a second set of Q fragments
  uint32_t pq[kPrefetchQ ? KC : 1][2];
  int pq_pos = -1;
  auto load_q = [&](const int4& r0, const int4& r2, auto& q) {
    const T* qrow = reinterpret_cast<const T*>(a.q) + (static_cast<size_t>(r0.x) * H + r2.z + gid) * D;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      q[kc][0] = gid < r2.w ? *reinterpret_cast<const uint32_t*>(qrow + kc * 16 + 2 * tig) : 0u;
      q[kc][1] = gid < r2.w ? *reinterpret_cast<const uint32_t*>(qrow + kc * 16 + 8 + 2 * tig) : 0u;
    }
  };
  // One step of the background fetch of the next unit.
  auto next_step = [&]() {
    if (n_state == 0) {
      if (lane == 0) n_ticket = atomicAdd(a.queue, 1u);  // used one step later
      n_state = 1;
    } else if (n_state == 1) {
      n_pos = W + static_cast<int>(__shfl_sync(0xffffffffu, n_ticket, 0));
      if (n_pos >= n_units) {
        n_state = 4;
        return;
      }
      const int4* rec = a.sched_recs + static_cast<size_t>(n_pos) * 3;
      n_r0 = rec[0];
      n_r1 = rec[1];
      n_r2 = rec[2];
      n_state = 2;
    } else if (n_state == 2) {
      load_pages(n_r0, n_r1, n_pg0, n_page0, n_page1);
      n_state = 3;
    }
  };
  bool dep_ready = false;  // the preceding kernel's results are visible (griddepcontrol.wait)
  auto start_unit = [&]() {
    p_j = p_r0.z / kSlab;
    p_end = (p_r0.w + kSlab - 1) / kSlab;
    // An empty context still gets one slab without data, so the consumer
    // finalizes the unit and writes its zero row (attention.hip:115).
    if (p_end <= p_j) p_end = p_j + 1;
    if constexpr (kPrefetchQ) {
      if (dep_ready) {  // q may come from the preceding kernel
        load_q(p_r0, p_r2, pq);
        pq_pos = p_pos;
      } else {
        pq_pos = -1;
      }
    }
  };
  // The first unit's record is plan data (never written by the preceding kernel);
  // its page ids come from the block tables, read before griddepcontrol.wait only
  // when they are declared stable.  The record is loaded while the unit count may
  // still be on its way (graph-stable plans read it from the device): sched_cap
  // bounds the load, the count decides whether the record is used.
  if (p_pos < a.sched_cap) {
    const int4* rec = a.sched_recs + static_cast<size_t>(p_pos) * 3;
    p_r0 = rec[0];
    p_r1 = rec[1];
    p_r2 = rec[2];
  }
  auto first_unit_pages = [&]() {
    if (p_pos < n_units) {
      load_pages(p_r0, p_r1, p_pg0, p_page0, p_page1);
      start_unit();
    }
  };
  if (a.early_prefetch) first_unit_pages();
  int issued = 0;
  auto p_issue = [&]() {  // all lanes; lane 0 issues the bulk copies
    while (p_j >= p_end) {  // current unit fully issued: move to the next one
      if (p_pos >= n_units) return;
      while (n_state < 3) next_step();
      if (n_state == 4) {
        p_pos = n_units;
        return;
      }
      p_pos = n_pos;
      p_r0 = n_r0;
      p_r1 = n_r1;
      p_r2 = n_r2;
      p_pg0 = n_pg0;
      p_page0 = n_page0;
      p_page1 = n_page1;
      n_state = 0;
      start_unit();
    }
    const int idx = p_j / spp - p_pg0;
    const int v0 = __shfl_sync(0xffffffffu, p_page0, idx & 31);
    const int v1 = __shfl_sync(0xffffffffu, p_page1, idx & 31);
    const int phys = p_r0.w > p_r0.z ? (idx < 32 ? v0 : v1) : -1;
    const int s = issued % NS;
    if (lane < 4) {
      int4 m = lane == 0 ? p_r0 : lane == 1 ? p_r1 : lane == 2 ? p_r2 : make_int4(phys, p_j, p_pos, 0);
      meta[s * 4 + lane] = m;
    }
    __syncwarp();
    if (lane == 0) {
      const uint32_t bar = smem_u32(&bars[s]);
      if (phys < 0) {
        mbar_arrive(bar);
      } else {
        const size_t off = static_cast<size_t>(phys) * page_stride +
                           static_cast<size_t>(p_r2.x) * ps * D * 2 +
                           static_cast<size_t>(p_j % spp) * SLAB_BYTES;
        mbar_arrive_expect_tx(bar, STAGE_BYTES);
        const uint32_t dst = smem_u32(stages + s * STAGE_BYTES);
        bulk_g2s(dst, a.k_layer + off, SLAB_BYTES, bar, policy);
        bulk_g2s(dst + SLAB_BYTES, a.v_layer + off, SLAB_BYTES, bar, policy);
      }
    }
    ++p_j;
    ++issued;
    next_step();
  };
  // Prologue: fill the ring.  Before griddepcontrol.wait only the plan, the
  // block tables and KV pages are read, and only when the caller declared them
  // stable across the preceding launch (KVC_PLAN_KV_STABLE); q, the new rows
  // and every write come after it.
  if (!a.early_prefetch) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    dep_ready = true;
    first_unit_pages();
  }
#pragma unroll 1
  for (int k = 0; k < NS; ++k) p_issue();
  if (!dep_ready) {
    // Still waiting for the preceding kernel (its merge, or the head exchange):
    // use the wait to bring the next l2_ahead slabs of this unit into L2, so
    // HBM streams during the wait and the ring later refills from L2.
    const int j = p_j + lane;
    const int idx = j / spp - p_pg0;
    const int v0 = __shfl_sync(0xffffffffu, p_page0, idx & 31);
    const int v1 = __shfl_sync(0xffffffffu, p_page1, idx & 31);
    if (lane < l2_ahead && p_pos < n_units && j < p_end && p_r0.w > p_r0.z) {
      const int phys = idx < 32 ? v0 : v1;
      if (phys >= 0) {
        const size_t off = static_cast<size_t>(phys) * page_stride +
                           static_cast<size_t>(p_r2.x) * ps * D * 2 +
                           static_cast<size_t>(j % spp) * SLAB_BYTES;
        bulk_prefetch_l2(a.k_layer + off, SLAB_BYTES);
        bulk_prefetch_l2(a.v_layer + off, SLAB_BYTES);
      }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    dep_ready = true;
  }

  // ---------------- consumer ----------------
  int consumed = 0, waited = 0;
  int cur = -1;  // list position of the unit being consumed
  int4 c_r0 = make_int4(0, 0, 0, 0), c_r1 = c_r0, c_r2 = c_r0;
  uint32_t qa[KC][2];
  float m_run = kNegBig, l_run = 0.f;
  float o[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  // End of a unit: the output row, or the split's partial state.
  auto finalize = [&]() {
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    const int query = c_r0.x, split = c_r0.y;
    const int slot0 = c_r1.z, n_splits = c_r1.w;
    const int hq0 = c_r2.z, nh = c_r2.w;
    // q-heads 2tig, 2tig+1 of this lane's O^T columns: their sums live in lanes 8tig, 8tig+4
    const float l_lo = __shfl_sync(0xffffffffu, l_run, (2 * tig) * 4);
    const float l_hi = __shfl_sync(0xffffffffu, l_run, (2 * tig + 1) * 4);
    const int h_lo = 2 * tig, h_hi = 2 * tig + 1;
    if (n_splits == 1 && a.xchg_peers == 0) {  // exchanged outputs all go through the merge
      const float i_lo = l_lo > 0.f ? 1.0f / l_lo : 0.f;
      const float i_hi = l_hi > 0.f ? 1.0f / l_hi : 0.f;
      T* out = reinterpret_cast<T*>(a.out) + (static_cast<size_t>(query) * H + hq0) * D;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (h_lo < nh) {
          out[h_lo * D + 16 * mt + gid] = from_f32<T>(o[mt][0] * i_lo);
          out[h_lo * D + 16 * mt + gid + 8] = from_f32<T>(o[mt][2] * i_lo);
        }
        if (h_hi < nh) {
          out[h_hi * D + 16 * mt + gid] = from_f32<T>(o[mt][1] * i_hi);
          out[h_hi * D + 16 * mt + gid + 8] = from_f32<T>(o[mt][3] * i_hi);
        }
      }
      return;
    }
    const size_t slot = static_cast<size_t>(slot0 + split) * H + hq0;
    float* po = a.part_o + slot * D;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      if (h_lo < nh) {
        po[h_lo * D + 16 * mt + gid] = o[mt][0];
        po[h_lo * D + 16 * mt + gid + 8] = o[mt][2];
      }
      if (h_hi < nh) {
        po[h_hi * D + 16 * mt + gid] = o[mt][1];
        po[h_hi * D + 16 * mt + gid + 8] = o[mt][3];
      }
    }
    if (tig == 0 && gid < nh) a.part_ml[slot + gid] = make_float2(m_run, l_run);
  };

  constexpr int K2 = D / 32;
  constexpr bool kAllFragsFirst = D <= 128;  // registers allow holding a whole slab
  bool dead = false;  // a wait ran past its limit: stop computing
#pragma unroll 1
  while (consumed < issued && !dead) {
    const int s = consumed % NS;
    const bool ok = mbar_wait_bounded(smem_u32(&bars[s]), static_cast<uint32_t>(consumed / NS) & 1u);
    if (__any_sync(0xffffffffu, !ok)) {
      if (lane == 0) report_error(2u /*KVC_DEVERR_WAIT_LIMIT*/, static_cast<uint32_t>(consumed));
      dead = true;
      break;
    }
    waited = consumed + 1;
    const int4 r3 = meta[s * 4 + 3];  // {phys, slab, list position}
    if (r3.z != cur) {
      if (cur >= 0) finalize();
      cur = r3.z;
      c_r0 = meta[s * 4 + 0];
      c_r1 = meta[s * 4 + 1];
      c_r2 = meta[s * 4 + 2];
      bool have_q = false;
      if constexpr (kPrefetchQ) {
        if (pq_pos == cur) {
#pragma unroll
          for (int kc = 0; kc < KC; ++kc) {
            qa[kc][0] = pq[kc][0];
            qa[kc][1] = pq[kc][1];
          }
          have_q = true;
        }
      }
      if (!have_q) load_q(c_r0, c_r2, qa);
      m_run = kNegBig;
      l_run = 0.f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      const int ctx = c_r1.y;
      if (a.k_new != nullptr && ctx > 0 && c_r0.w == ctx && c_r2.y == 0)
        append_row_to_pool(a, kLayoutCore, 2, c_r0.x, c_r2.x, ctx - 1,
                           a.block_tables + static_cast<size_t>(c_r1.x) * a.bt_stride, lane);
    }
    const int j = r3.y;
    const int te = c_r0.w, ctx = c_r1.y;
    const bool have = r3.x >= 0;
    const int valid = min(kSlab, te - j * kSlab);
    uint8_t* st = stages + s * STAGE_BYTES;
    const uint32_t kbase = smem_u32(st);
    const uint32_t vbase = kbase + SLAB_BYTES;
    const int jm = lane >> 3;
    if (have) {
      if (valid < kSlab) {
        // positions past the context may hold anything: clear them
        const int nunits = (kSlab - valid) * U;
        for (int x = lane; x < 2 * nunits; x += 32) {
          const int kv = x / nunits, r = x - kv * nunits;
          const int tt = valid + r / U, uu = r - (r / U) * U;
          *reinterpret_cast<uint4*>(st + kv * SLAB_BYTES + unit_offset(kLayoutCore, tt, uu, U) * 16) =
              make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      if (a.k_new != nullptr && ctx > 0 && te == ctx && j == (ctx - 1) / kSlab) {
        patch_slab_row(a, kLayoutCore, 2, st, SLAB_BYTES, c_r0.x, c_r2.x, (ctx - 1) - j * kSlab,
                       lane, 32);
        __syncwarp();
      }
    }
    // K and V fragments of the slab (all of them when registers allow, so the
    // stage can be refilled before the math; otherwise K first, V after S).
    constexpr int KF = kAllFragsFirst ? K2 : 1;
    uint32_t kf[KF][2][4];
    uint32_t vf[kAllFragsFirst ? MT : 1][4];
    float sc[2][2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int par = 0; par < 2; ++par)
        sc[nt][par][0] = sc[nt][par][1] = sc[nt][par][2] = sc[nt][par][3] = 0.f;
    if (have) {
      if constexpr (kAllFragsFirst) {
#pragma unroll
        for (int k2 = 0; k2 < K2; ++k2)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
            ldsm_x4(kbase + ((nt * U + k2 * 4 + (lane >> 3)) * 8 + (lane & 7)) * 16, kf[k2][nt][0],
                    kf[k2][nt][1], kf[k2][nt][2], kf[k2][nt][3]);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          ldsm_x4_t(vbase + (((jm >> 1) * U + 2 * mt + (jm & 1)) * 8 + (lane & 7)) * 16, vf[mt][0],
                    vf[mt][1], vf[mt][2], vf[mt][3]);
      }
#pragma unroll
      for (int k2 = 0; k2 < K2; ++k2) {
        const int kk = kAllFragsFirst ? k2 : 0;
        if constexpr (!kAllFragsFirst) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
            ldsm_x4(kbase + ((nt * U + k2 * 4 + (lane >> 3)) * 8 + (lane & 7)) * 16, kf[0][nt][0],
                    kf[0][nt][1], kf[0][nt][2], kf[0][nt][3]);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          Mma<T>::run(sc[nt][0], qa[2 * k2][0], 0u, qa[2 * k2][1], 0u, kf[kk][nt][0], kf[kk][nt][1]);
          Mma<T>::run(sc[nt][1], qa[2 * k2 + 1][0], 0u, qa[2 * k2 + 1][1], 0u, kf[kk][nt][2],
                      kf[kk][nt][3]);
        }
      }
    }
    if constexpr (kAllFragsFirst) {
      // Every fragment has landed in registers (the XOR reads one register of
      // each ldmatrix, so it waits for all of them): the stage can be refilled
      // before the math.
      uint32_t dep = 0;
      if (have) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) dep ^= vf[mt][0];
      }
      asm volatile("" ::"r"(dep));
      __syncwarp();
      ++consumed;
      if (lane == 0) fence_proxy_async();
      p_issue();
    }
    if (!have) {
      if constexpr (!kAllFragsFirst) {
        __syncwarp();
        ++consumed;
        if (lane == 0) fence_proxy_async();
        p_issue();
      }
      continue;
    }

    const int t0 = 2 * tig;
    const bool v0 = t0 < valid, v1 = t0 + 1 < valid, v2 = t0 + 8 < valid, v3 = t0 + 9 < valid;
    const float x0 = (sc[0][0][0] + sc[0][1][0]) * a.scale_log2;
    const float x1 = (sc[0][0][1] + sc[0][1][1]) * a.scale_log2;
    const float x2 = (sc[1][0][0] + sc[1][1][0]) * a.scale_log2;
    const float x3 = (sc[1][0][1] + sc[1][1][1]) * a.scale_log2;
    float mx = fmaxf(fmaxf(v0 ? x0 : kNegBig, v1 ? x1 : kNegBig),
                     fmaxf(v2 ? x2 : kNegBig, v3 ? x3 : kNegBig));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float alpha = fast_exp2(m_run - m_new);
    const float p0 = v0 ? fast_exp2(x0 - m_new) : 0.f;
    const float p1 = v1 ? fast_exp2(x1 - m_new) : 0.f;
    const float p2 = v2 ? fast_exp2(x2 - m_new) : 0.f;
    const float p3 = v3 ? fast_exp2(x3 - m_new) : 0.f;
    l_run = l_run * alpha + ((p0 + p1) + (p2 + p3));
    m_run = m_new;
    const uint32_t pb0 = Mma<T>::pack(p0, p1);
    const uint32_t pb1 = Mma<T>::pack(p2, p3);
    const float a_lo = __shfl_sync(0xffffffffu, alpha, (2 * tig) * 4);
    const float a_hi = __shfl_sync(0xffffffffu, alpha, (2 * tig + 1) * 4);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      o[mt][0] *= a_lo;
      o[mt][1] *= a_hi;
      o[mt][2] *= a_lo;
      o[mt][3] *= a_hi;
      if constexpr (kAllFragsFirst) {
        Mma<T>::run(o[mt], vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3], pb0, pb1);
      } else {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vbase + (((jm >> 1) * U + 2 * mt + (jm & 1)) * 8 + (lane & 7)) * 16, r0, r1, r2,
                  r3);
        Mma<T>::run(o[mt], r0, r1, r2, r3, pb0, pb1);
      }
    }
    if constexpr (!kAllFragsFirst) {  // the stage is released after the math
      __syncwarp();
      ++consumed;
      if (lane == 0) fence_proxy_async();
      p_issue();
    }
  }
  if (cur >= 0 && !dead) finalize();
  // Bounded waits for copies still landing in this warp's ring (none unless a
  // wait gave up above).
  for (int k = waited; k < issued; ++k)
    (void)mbar_wait_bounded(smem_u32(&bars[k % NS]), static_cast<uint32_t>(k / NS) & 1u);
  // The split merge (a programmatic dependent launch) may start being scheduled.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// =====================================================================================
// Split merge of the persistent path.  Runs as a programmatic dependent launch
// after decode_persistent_kernel and waits for it (griddepcontrol.wait) before
// reading the partial states:
//   M = max_k M_k,  L = sum_k L_k 2^(M_k - M),  out = sum_k O_k 2^(M_k - M) / L
// One CTA of kMergeWarps (8) warps serves 8 / WPH q-heads of one query.  The WPH warps of a
// head take contiguous ranges of its splits; each warp merges its range in one
// pass (running maximum per 32 splits, eight splits' loads in flight), and the
// ranges are then combined in range order through shared memory.  The order of
// every addition is fixed, so the result does not depend on timing, and a long
// context with few queries (hundreds of splits per head) merges in a few memory
// round trips.
// =====================================================================================
template <typename T, int EPL>
__global__ void __launch_bounds__(32 * kMergeWarps) merge_splits_kernel(const DecodeArgs a) {
  __shared__ float red_acc[kMergeWarps][EPL * 32];
  __shared__ float red_m[kMergeWarps], red_l[kMergeWarps];
  const bool xchg = a.xchg_peers > 0;
  // Counts: from the launch, or from the plan's device header for a graph-stable
  // plan, whose grid is sized for the most CTAs any of its rebuilds can need
  // (n_queries x num_heads); the CTAs a rebuild does not need leave at once
  // (CTA (0, 0) always stays: it re-arms the unit counter).
  // The query's record is plan data, which the decode grid does not write: read
  // it before the wait, so only the partials' loads follow the decode's end.
  // exchanged outputs: every query (grid.x = n_queries); else the multi-split ones
  int n_merge = a.n_merge_queries, wph = a.merge_wph;
  int query = 0;
  int4 qi = make_int4(0, 0, 0, 0);
  if (a.plan_hdr) {
    // the counts, this CTA's list entry and its query's record, all loads at once
    // (the list has a slot per query; an entry past the count may be stale, so
    // it is clamped and its record used only when the CTA turns out to be needed)
    n_merge = a.plan_hdr[kHdrMergeQueries];
    wph = a.plan_hdr[kHdrMergeWph];
    query = xchg ? static_cast<int>(blockIdx.x) : a.merge_queries[blockIdx.x];
    query = min(max(query, 0), a.n_queries_total - 1);
    qi = a.qinfo[query];
  }
  const int heads_per_cta = kMergeWarps / wph;
  const bool mine = (xchg || static_cast<int>(blockIdx.x) < n_merge) &&
                    static_cast<int>(blockIdx.y) * heads_per_cta < a.num_heads;
  if (!mine && (blockIdx.x | blockIdx.y) != 0) return;
  if (mine && !a.plan_hdr) {
    query = xchg ? static_cast<int>(blockIdx.x) : a.merge_queries[blockIdx.x];
    qi = a.qinfo[query];
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The decode grid has finished: re-arm its unit counter for the next launch,
  // visibly to the whole device before the next launch may start, and copy the
  // device error word (every error of the decode is in it now) to its host mirror.
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    *a.queue = 0u;
    if (uint32_t* m = a.err_host) {
      const volatile uint32_t* w = g_kvc_deverr;
      m[1] = w[1];
      m[0] = w[0];
    }
    __threadfence();
  }
  __syncthreads();
  // the next decode launch may start filling its ring while the merge runs
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!mine) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = warp % wph;                  // wph: 1, 2, 4 or 8
  const int h = blockIdx.y * heads_per_cta + warp / wph;
  const bool active = h < a.num_heads;
  const int H = a.num_heads, D = a.head_dim;
  float m_run = kNegBig, sum = 0.f;
  float acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
  if (active) {
    const int slot0 = qi.z, n = qi.w;
    const float2* ml = a.part_ml + static_cast<size_t>(slot0) * H + h;
    const float* po = a.part_o + (static_cast<size_t>(slot0) * H + h) * D + lane;
    // this warp's range of splits
    const int per = (n + wph - 1) / wph;
    const int kb = min(n, sub * per), ke = min(n, kb + per);
    for (int k0 = kb; k0 < ke; k0 += 32) {
      const int kn = min(32, ke - k0);
      float2 st = make_float2(kNegBig, 0.f);
      if (lane < kn) st = __ldcg(&ml[static_cast<size_t>(k0 + lane) * H]);
      float cm = st.x;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      if (cm > m_run) {  // warp-uniform: rescale what this warp has so far
        const float r = fast_exp2(m_run - cm);
        sum *= r;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] *= r;
        m_run = cm;
      }
      const float w = lane < kn ? fast_exp2(st.x - m_run) : 0.f;
      sum += st.y * w;
      // eight splits' loads in flight at once; the batch past the range's end
      // loads nothing and adds zeros
      for (int kk = 0; kk < kn; kk += 8) {
        float v[8][EPL];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const bool ok = kk + u < kn;
#pragma unroll
          for (int e = 0; e < EPL; ++e)
            v[u][e] = ok ? __ldcg(po + static_cast<size_t>(k0 + kk + u) * H * D + 32 * e) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float wk = __shfl_sync(0xffffffffu, w, (kk + u) & 31);
          wk = kk + u < kn ? wk : 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) acc[e] += v[u][e] * wk;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  if (wph > 1) {  // combine the ranges of a head in order
#pragma unroll
    for (int e = 0; e < EPL; ++e) red_acc[warp][32 * e + lane] = acc[e];
    if (lane == 0) {
      red_m[warp] = m_run;
      red_l[warp] = sum;
    }
    __syncthreads();
    if (sub == 0 && active) {
      float mx = m_run;
      for (int j = 1; j < wph; ++j) mx = fmaxf(mx, red_m[warp + j]);
      const float r0 = fast_exp2(m_run - mx);
      sum *= r0;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] *= r0;
      for (int j = 1; j < wph; ++j) {
        const float r = fast_exp2(red_m[warp + j] - mx);
        sum += red_l[warp + j] * r;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] += red_acc[warp + j][32 * e + lane] * r;
      }
    }
  }
  if (sub == 0 && active) {
    const float inv = sum > 0.f ? 1.0f / sum : 0.f;
    if (!xchg) {
      T* out = reinterpret_cast<T*>(a.out) + (static_cast<size_t>(query) * H + h) * D + lane;
#pragma unroll
      for (int e = 0; e < EPL; ++e) out[32 * e] = from_f32<T>(acc[e] * inv);
    } else {
      // the row goes to every rank's exchange slot (this rank's included)
      const size_t off = (static_cast<size_t>(query) * a.out_heads + a.out_head0 + h) * D + lane;
      T val[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) val[e] = from_f32<T>(acc[e] * inv);
      for (int p = 0; p < a.xchg_peers; ++p) {
        T* out = reinterpret_cast<T*>(a.peer_out[p]) + off;
#pragma unroll
        for (int e = 0; e < EPL; ++e) out[32 * e] = val[e];
      }
    }
  }
}

// Exchange completion, one warp after the merge grid (programmatic dependent
// launch).  griddepcontrol.wait returns when the merge grid has finished and its
// stores (this rank's heads, already written into every rank's slot) are
// performed; one system-scope acq_rel fence then orders them before the epoch this rank
// publishes in its flag word on every rank, and lane p waits (bounded) until
// rank p has published the same epoch here.  Only other GPUs' kernels are
// waited for.  The epoch is one more than this rank's previous one, kept on the
// device so a captured graph replays with fresh epochs; every rank makes the
// same sequence of exchanges, so the counters agree.
__global__ void __launch_bounds__(32) xchg_signal_kernel(const DecodeArgs a) {
  // the next decode launch may be scheduled while this waits
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x;
  unsigned epoch = 0;
  if (lane == 0) {
    epoch = *a.epoch_ctr + 1u;
    *a.epoch_ctr = epoch;
    // release pattern: one acq_rel fence at system scope, then relaxed flag stores
    fence_acq_rel_sys();
    for (int p = 0; p < a.xchg_peers; ++p) st_relaxed_sys(a.peer_flag[p], epoch);
  }
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  if (lane >= a.xchg_peers) return;
  const unsigned long long t0 = globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys(a.my_flags + lane) - epoch) < 0) {
    if (globaltimer_ns() - t0 > a.wait_limit_ns) {
      report_error(2u /*KVC_DEVERR_WAIT_LIMIT*/, 0x10000u + static_cast<uint32_t>(lane));
      return;
    }
    __nanosleep(64);
  }
}

// =====================================================================================
// CUDA-core split-K decode kernel: fp32 storage (linear layout) and 16-bit head
// dims the tensor-core kernel does not cover.  One warp per q-head of the chunk,
// lanes over head dims (element d = lane + 32 e, like attention.hip:65-73), the
// CTA streams slabs through an NS-deep ring filled by thread 0.
// =====================================================================================
template <typename T, int EPL, int NS>
__global__ void __launch_bounds__(256) decode_simt_kernel(const DecodeArgs a, int layout) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int D = a.head_dim;
  const int ES = static_cast<int>(sizeof(T));
  const int U = D * ES / 16;
  const int slab_bytes = kSlab * D * ES;
  const int stage_bytes = 2 * slab_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int b = blockIdx.x;
  const int hc = b % a.n_hchunk;
  b /= a.n_hchunk;
  const int kvh = b % a.num_kv_heads;
  b /= a.num_kv_heads;
  const int4 it = a.items[2 * b];
  const int4 qi = a.items[2 * b + 1];
  const int query = it.x, split = it.y, tb = it.z, te = it.w;
  const int hq0 = kvh * a.group + hc * 8;
  const int nh = min(8, a.group - hc * 8);
  const int ps = a.page_size;
  const int slabs_per_page = ps / kSlab;
  const bool active = warp < nh;

  uint8_t* const region = smem + kBarBytes;  // [mbarriers] [NS stages], reused by the merge
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncthreads();

  float q[EPL], acc[EPL];
  {
    const T* qrow = reinterpret_cast<const T*>(a.q) +
                    (static_cast<size_t>(query) * a.num_heads + hq0 + (active ? warp : 0)) * D;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane + 32 * e;
      q[e] = (active && d < D) ? to_f32<T>(qrow[d]) : 0.f;
      acc[e] = 0.f;
    }
  }

  const int sb0 = tb / kSlab;
  const int nslabs = (te + kSlab - 1) / kSlab - sb0;
  const int32_t* bt_row = a.block_tables + static_cast<size_t>(qi.x) * a.bt_stride;
  const size_t head_off = static_cast<size_t>(kvh) * ps * D * ES;
  const size_t page_stride = static_cast<size_t>(a.num_kv_heads) * ps * D * ES;
  const uint64_t policy = l2_policy_evict_first();

  // The split's page ids, read once into shared memory.
  __shared__ int s_pages[kMaxSplitPages];
  const int pg0 = tb / ps;
  const int npages = (te + ps - 1) / ps - pg0;
  if (threadIdx.x < kMaxSplitPages) {
    int v = -1;
    if (static_cast<int>(threadIdx.x) < npages) {
      v = pg0 + static_cast<int>(threadIdx.x) < a.bt_stride ? bt_row[pg0 + threadIdx.x] : -1;
      if (v < 0 || v >= a.num_pages) {
        report_error(1u, static_cast<uint32_t>(v));
        v = -1;
      }
    }
    s_pages[threadIdx.x] = v;
  }
  __syncthreads();
  auto slab_page = [&](int j) -> int { return s_pages[j / slabs_per_page - pg0]; };
  auto issue = [&](int i) {  // thread 0 only
    const int j = sb0 + i;
    const int s = i % NS;
    const uint32_t bar = smem_u32(&bars[s]);
    const int phys = slab_page(j);
    if (phys < 0) {
      mbar_arrive(bar);
      return;
    }
    const size_t off = static_cast<size_t>(phys) * page_stride + head_off +
                       static_cast<size_t>(j % slabs_per_page) * slab_bytes;
    mbar_arrive_expect_tx(bar, stage_bytes);
    const uint32_t dst = smem_u32(region + s * stage_bytes);
    bulk_g2s(dst, a.k_layer + off, slab_bytes, bar, policy);
    bulk_g2s(dst + slab_bytes, a.v_layer + off, slab_bytes, bar, policy);
  };

  if (threadIdx.x == 0)
    for (int i = 0; i < min(NS, nslabs); ++i) issue(i);
  int issued = min(NS, nslabs);

  const int ctx = qi.y;
  const bool owns_new = a.k_new != nullptr && ctx > 0 && te == ctx;
  const int new_slab = (ctx - 1) / kSlab;
  if (owns_new && hc == 0 && warp == 0)
    append_row_to_pool(a, layout, ES, query, kvh, ctx - 1, bt_row, lane);

  float m_run = kNegBig, l_run = 0.f;
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  __syncthreads();
  int consumed = 0;
  for (int i = 0; i < nslabs; ++i) {
    const int s = i % NS;
    const int j = sb0 + i;
    if (!mbar_wait_bounded(smem_u32(&bars[s]), static_cast<uint32_t>(i / NS) & 1u)) {
      if (threadIdx.x == 0) report_error(2u, static_cast<uint32_t>(j));
      s_abort = 1;
    }
    __syncthreads();
    if (s_abort) break;
    consumed = i + 1;
    const uint8_t* st = region + s * stage_bytes;
    const int valid = min(kSlab, te - j * kSlab);
    if (owns_new && j == new_slab) {
      patch_slab_row(a, layout, ES, const_cast<uint8_t*>(st), slab_bytes, query, kvh,
                     (ctx - 1) - j * kSlab, threadIdx.x, blockDim.x);
      __syncthreads();
    }
    if (active && slab_page(j) >= 0) {
      for (int t = 0; t < valid; ++t) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const int d = lane + 32 * e;
          if (d < D) {
            const T* kp = reinterpret_cast<const T*>(
                st + unit_offset(layout, t, (d * ES) >> 4, U) * 16 + ((d * ES) & 15));
            dot += q[e] * to_f32<T>(*kp);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float x = dot * a.scale_log2;
        const float m_new = fmaxf(m_run, x);
        const float alpha = fast_exp2(m_run - m_new);
        const float p = fast_exp2(x - m_new);
        l_run = l_run * alpha + p;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const int d = lane + 32 * e;
          if (d < D) {
            const T* vp = reinterpret_cast<const T*>(
                st + slab_bytes + unit_offset(layout, t, (d * ES) >> 4, U) * 16 + ((d * ES) & 15));
            acc[e] = acc[e] * alpha + p * to_f32<T>(*vp);
          }
        }
        m_run = m_new;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && i + NS < nslabs) {
      fence_proxy_async();
      issue(i + NS);
    }
    if (i + NS < nslabs) issued = i + NS + 1;
  }
  if (threadIdx.x == 0)
    for (int i = consumed; i < issued; ++i)
      (void)mbar_wait_bounded(smem_u32(&bars[i % NS]), static_cast<uint32_t>(i / NS) & 1u);
  __syncthreads();

  const int n_splits = qi.w;
  const int H = a.num_heads;
  if (active) {
    const int h = warp;
    if (n_splits == 1) {
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      T* out = reinterpret_cast<T*>(a.out) + (static_cast<size_t>(query) * H + hq0 + h) * D;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const int d = lane + 32 * e;
        if (d < D) out[d] = from_f32<T>(acc[e] * inv);
      }
    } else {
      const size_t slot = static_cast<size_t>(qi.z + split) * H + hq0 + h;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const int d = lane + 32 * e;
        if (d < D) a.part_o[slot * D + d] = acc[e];
      }
      if (lane == 0) a.part_ml[slot] = make_float2(m_run, l_run);
    }
  }
  if (n_splits > 1) {
    __syncthreads();
    finish_split<T>(a, reinterpret_cast<float*>(region), query, kvh, hc, qi.z, n_splits, hq0, nh);
  }
}

// =====================================================================================
// Host-side dispatch.
// =====================================================================================
namespace {

// Dynamic shared memory opt-in, once per kernel, device and size (it is not a
// stream operation, and skipping it keeps launches cheap and capture-safe).
constexpr int kMaxDevices = 64;
template <auto Kernel, typename F>
cudaError_t set_smem_once(F kern, size_t smem) {
  static std::atomic<size_t> done[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire) >= smem)
    return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
  if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    size_t cur = done[dev].load(std::memory_order_relaxed);
    while (cur < smem && !done[dev].compare_exchange_weak(cur, smem)) {
    }
  }
  return e;
}

template <typename T, int D, int NW>
cudaError_t run_persistent(const DecodeArgs& a, cudaStream_t s) {
  constexpr int NS = persist_stages<D>();
  const size_t smem =
      kPersistBarBytes + kPersistMetaBytes + static_cast<size_t>(NW) * NS * 2 * kSlab * D * 2;
  auto kern = decode_persistent_kernel<T, D, NW, NS>;
  cudaError_t e = set_smem_once<decode_persistent_kernel<T, D, NW, NS>>(kern, smem);
  if (e != cudaSuccess) return e;
  if (a.n_sched_ctas <= 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    // programmatic dependent launch: the ring prologue may overlap the tail of
    // the preceding kernel (see griddepcontrol.wait in the kernel)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.n_sched_ctas), 1, 1);
    cfg.blockDim = dim3(NW * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if ((e = cudaLaunchKernelEx(&cfg, kern, a)) != cudaSuccess) return e;
  }
  // merge (and counter re-arm) as a programmatic dependent launch: scheduled while
  // the decode grid drains
  cudaLaunchConfig_t cfg = {};
  if (a.plan_hdr) {
    // graph-stable plan: room for every query and one q-head per CTA (the most
    // any rebuild of the plan can use); the kernel reads the counts
    cfg.gridDim = dim3(static_cast<unsigned>(a.n_queries_total > 0 ? a.n_queries_total : 1),
                       static_cast<unsigned>(a.num_heads), 1);
  } else {
    const int n_merge = a.xchg_peers > 0 ? a.n_queries_total : a.n_merge_queries;
    const int heads_per_cta = kMergeWarps / a.merge_wph;
    cfg.gridDim = dim3(static_cast<unsigned>(n_merge > 0 ? n_merge : 1),
                       n_merge > 0 ? (a.num_heads + heads_per_cta - 1) / heads_per_cta : 1, 1);
  }
  cfg.blockDim = dim3(32 * kMergeWarps, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if ((e = cudaLaunchKernelEx(&cfg, merge_splits_kernel<T, D / 32>, a)) != cudaSuccess) return e;
  if (a.xchg_peers == 0) return cudaSuccess;
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  return cudaLaunchKernelEx(&cfg, xchg_signal_kernel, a);
}

template <typename T, int D>
cudaError_t run_mma(const DecodeArgs& a, cudaStream_t s) {
  return run_persistent<T, D, kPersistWarps>(a, s);
}

template <typename T, int EPL>
cudaError_t run_simt(const DecodeArgs& a, int layout, cudaStream_t s) {
  constexpr int NS = 3;
  const size_t stage_bytes = 2 * static_cast<size_t>(kSlab) * a.head_dim * sizeof(T);
  size_t smem = NS * stage_bytes;
  const size_t merge = (8 * kMergeChunk + 8 * static_cast<size_t>(a.head_dim) + 16) * sizeof(float);
  if (merge > smem) smem = merge;
  smem += kBarBytes;
  auto kern = decode_simt_kernel<T, EPL, NS>;
  cudaError_t e = set_smem_once<decode_simt_kernel<T, EPL, NS>>(kern, smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(a.n_items) * a.num_kv_heads * a.n_hchunk;
  kern<<<grid, 256, smem, s>>>(a, layout);
  return cudaGetLastError();
}

template <typename T>
cudaError_t run_simt_any(const DecodeArgs& a, int layout, cudaStream_t s) {
  const int epl = (a.head_dim + 31) / 32;
  if (epl <= 1) return run_simt<T, 1>(a, layout, s);
  if (epl <= 2) return run_simt<T, 2>(a, layout, s);
  if (epl <= 4) return run_simt<T, 4>(a, layout, s);
  return run_simt<T, 8>(a, layout, s);
}

template <typename T>
cudaError_t run_mma_any(const DecodeArgs& a, cudaStream_t s) {
  switch (a.head_dim) {
    case 32: return run_mma<T, 32>(a, s);
    case 64: return run_mma<T, 64>(a, s);
    case 96: return run_mma<T, 96>(a, s);
    case 128: return run_mma<T, 128>(a, s);
    case 160: return run_mma<T, 160>(a, s);
    case 192: return run_mma<T, 192>(a, s);
    case 256: return run_mma<T, 256>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool decode_uses_mma(int dtype, int head_dim, int page_size) {
  if (dtype != 0 && dtype != 1) return false;
  if (page_size % kSlab != 0) return false;
  switch (head_dim) {
    case 32: case 64: case 96: case 128: case 160: case 192: case 256: return true;
    default: return false;
  }
}

cudaError_t launch_decode(const DecodeArgs& a, int dtype, int layout, cudaStream_t s) {
  if (a.n_items == 0) return cudaSuccess;
  if (decode_uses_mma(dtype, a.head_dim, a.page_size) && layout == kLayoutCore) {
    return dtype == 1 ? run_mma_any<__nv_bfloat16>(a, s) : run_mma_any<__half>(a, s);
  }
  if (dtype == 2) return run_simt_any<float>(a, layout, s);
  if (dtype == 1) return run_simt_any<__nv_bfloat16>(a, layout, s);
  return run_simt_any<__half>(a, layout, s);
}

}  // namespace kvc

// =====================================================================================
// kvc_decode_noalloc: the decode for callers that cannot allocate device memory.
//
// Some hosts of this library (a runtime that owns every device allocation
// through its own arena, a plugin that may not call cudaMalloc) can still hand
// over their KV pages, q and out, but cannot let the library allocate its plan
// and split scratch.  This entry point keeps both in g_noalloc_scratch, a
// file-scope device array of kNoAllocScratchBytes that every GPU loading the
// library holds until the process exits, and stages the plan in static host
// buffers.  It calls no cudaMalloc / cudaFree or other allocating routine.
// Requests that do not fit are rejected with KVC_ERR_INVALID_ARG, and so is a
// call on a stream that is being captured (the plan is uploaded from pageable
// host memory, which a capture cannot record).
// =====================================================================================


namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB per device
constexpr int kNoAllocMaxQueries = 4096;
constexpr int kNoAllocMaxItems = 16384;
constexpr int kNoAllocMaxUnits = 65536;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;

// Host staging (static, no heap).  Layout mirrors the device scratch.
int4 h_items[kNoAllocMaxItems];
int4 h_qinfo[kNoAllocMaxQueries];
int4 h_recs[3 * kNoAllocMaxUnits];
int32_t h_merge[kNoAllocMaxQueries];
int h_refine[kNoAllocMaxQueries];
int32_t h_order[kNoAllocMaxItems];
int4 h_item_pairs[2 * kNoAllocMaxItems];

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

extern "C" int kvc_decode_noalloc(const void* d_k_layer, const void* d_v_layer, int num_pages,
                                  int page_size, int num_kv_heads, int head_dim, int dtype,
                                  const int32_t* d_block_tables, int bt_stride,
                                  const int32_t* h_ctx_lens, int n_queries, int num_heads,
                                  const void* d_q, void* d_out, float scale, void* stream) {
  using namespace kvc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (dtype != KVC_DTYPE_F16 && dtype != KVC_DTYPE_BF16)
    return set_error(KVC_ERR_INVALID_ARG, "kvc_decode_noalloc supports fp16 and bf16 KV pages only.");
  if (!decode_uses_mma(dtype, head_dim, page_size))
    return set_error(KVC_ERR_INVALID_ARG,
                     "kvc_decode_noalloc needs head_dim in {32,64,96,128,160,192,256} and a "
                     "page_size multiple of 16 (got %d, %d).", head_dim, page_size);
  if (num_pages <= 0 || num_kv_heads <= 0 || bt_stride <= 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_pages, num_kv_heads and bt_stride must be positive.");
  if (num_heads <= 0 || num_heads % num_kv_heads != 0)
    return set_error(KVC_ERR_INVALID_ARG, "num_heads must be divisible by num_kv_heads.");
  if (n_queries < 0 || n_queries > kNoAllocMaxQueries)
    return set_error(KVC_ERR_INVALID_ARG, "kvc_decode_noalloc accepts at most %d queries (got %d).",
                     kNoAllocMaxQueries, n_queries);
  if (n_queries == 0) return KVC_OK;
  if (!d_k_layer || !d_v_layer || !d_block_tables || !h_ctx_lens || !d_q || !d_out)
    return set_error(KVC_ERR_INVALID_ARG, "pointers must not be null.");
  if ((reinterpret_cast<uintptr_t>(d_k_layer) | reinterpret_cast<uintptr_t>(d_v_layer)) & 15u)
    return set_error(KVC_ERR_INVALID_ARG, "KV page buffers must be 16-byte aligned.");
  if ((reinterpret_cast<uintptr_t>(d_q) | reinterpret_cast<uintptr_t>(d_out)) & 3u)
    return set_error(KVC_ERR_INVALID_ARG, "q and out must be 4-byte aligned.");

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Before any other CUDA call: a capturing stream is refused without touching it
  // (the capture stays valid).
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &cap);
  if (e != cudaSuccess) return cuda_error(e, "cudaStreamIsCapturing");
  if (cap != cudaStreamCaptureStatusNone)
    return set_error(KVC_ERR_INVALID_ARG,
                     "kvc_decode_noalloc cannot run on a stream that is being captured: its plan "
                     "is uploaded from pageable host memory.");
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  // The device address of the scratch array on the current device (its host-side
  // name is only a stand-in, not a device pointer).  Looked up on every call: the
  // lookup allocates nothing, and a call after cudaDeviceReset finds the array at
  // its new address.
  void* scratch = nullptr;
  if ((e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch)) != cudaSuccess)
    return cuda_error(e, "cudaGetSymbolAddress(noalloc scratch)");

  // ---- split list: the same partition as kvc_plan_decode ----
  for (int i = 0; i < n_queries; ++i) {
    if (h_ctx_lens[i] < 0)
      return set_error(KVC_ERR_INVALID_ARG, "context length must be non-negative.");
    if (static_cast<int64_t>(h_ctx_lens[i]) > static_cast<int64_t>(bt_stride) * page_size)
      return set_error(KVC_ERR_OUT_OF_RANGE, "a context length exceeds the block-table width.");
  }
  const int C = split_partition(page_size, h_ctx_lens, n_queries,
                                num_kv_heads * ((num_heads / num_kv_heads + 7) / 8), dev, h_refine);
  int n_items = 0, slot = 0, max_splits = 0;
  for (int i = 0; i < n_queries; ++i) {
    const int ctx = h_ctx_lens[i];
    const int base = ctx > 0 ? (ctx + C - 1) / C : 1;
    if (n_items + base + 3 * h_refine[i] > kNoAllocMaxItems)
      return set_error(KVC_ERR_INVALID_ARG, "kvc_decode_noalloc accepts at most %d splits.",
                       kNoAllocMaxItems);
    const int ns = emit_splits(i, ctx, C, h_refine[i], [&](const int4& it) { h_items[n_items++] = it; });
    h_qinfo[i] = make_int4(i, ctx, slot, ns);
    slot += ns;
    max_splits = std::max(max_splits, ns);
  }
  for (int k = 0; k < n_items; ++k) h_order[k] = k;
  std::sort(h_order, h_order + n_items, [](int x, int y) {
    const int lx = h_items[x].w - h_items[x].z, ly = h_items[y].w - h_items[y].z;
    return lx != ly ? lx > ly : x < y;
  });
  const int group = num_heads / num_kv_heads;
  const int nhc = (group + 7) / 8;
  const int per_item = num_kv_heads * nhc;
  const int64_t n_units64 = static_cast<int64_t>(n_items) * per_item;
  if (n_units64 > kNoAllocMaxUnits)
    return set_error(KVC_ERR_INVALID_ARG, "kvc_decode_noalloc accepts at most %d work units.",
                     kNoAllocMaxUnits);
  const int n_units = static_cast<int>(n_units64);

  // ---- scratch layout and size check ----
  const size_t H = static_cast<size_t>(num_heads);
  const size_t off_queue = 0;
  const size_t off_items = 256;
  const size_t off_qinfo = align256(off_items + sizeof(int4) * 2 * n_items);
  const size_t off_recs = align256(off_qinfo + sizeof(int4) * n_queries);
  const int sms = device_sms(dev);
  const int n_ctas = std::max(1, std::min(sms * kPersistCtasPerSm,
                                          (n_units + kPersistWarps - 1) / kPersistWarps));
  const size_t off_merge = align256(off_recs + sizeof(int4) * 3 * n_units);
  const size_t plan_bytes = align256(off_merge + sizeof(int32_t) * n_queries);
  const size_t off_part_ml = plan_bytes;
  const size_t off_part_o = align256(off_part_ml + sizeof(float2) * slot * H);
  const size_t need = off_part_o + sizeof(float) * slot * H * head_dim;
  if (need > kNoAllocScratchBytes)
    return set_error(KVC_ERR_INVALID_ARG,
                     "kvc_decode_noalloc needs %zu bytes of scratch for this batch; its fixed "
                     "scratch holds %zu bytes (use kvc_decode for larger batches).",
                     need, kNoAllocScratchBytes);

  // ---- units, longest first (the kernel hands them out dynamically) ----
  for (int r = 0; r < n_units; ++r) {
    const int k = h_order[r / per_item];
    const int u = r % per_item;
    const int kvh = u / nhc, hc = u % nhc;
    const int4 it = h_items[k];
    h_recs[3 * r + 0] = it;
    h_recs[3 * r + 1] = h_qinfo[it.x];  // {bt row = query, ctx, slot0, n_splits}
    h_recs[3 * r + 2] = make_int4(kvh, hc, kvh * group + hc * 8, std::min(8, group - hc * 8));
  }
  int n_merge = 0;
  for (int i = 0; i < n_queries; ++i)
    if (h_qinfo[i].w > 1) h_merge[n_merge++] = i;
  for (int k = 0; k < n_items; ++k) {
    h_item_pairs[2 * k] = h_items[h_order[k]];
    h_item_pairs[2 * k + 1] = h_qinfo[h_items[h_order[k]].x];
  }

  // ---- upload (pageable host source: the call returns once it is staged) ----
  uint8_t* base = static_cast<uint8_t*>(scratch);
  // the unit counter starts at zero (this call's merge kernel re-arms it too)
  if ((e = cudaMemsetAsync(base + off_queue, 0, 256, s)))
    return cuda_error(e, "kvc_decode_noalloc counter reset");
  if ((e = cudaMemcpyAsync(base + off_items, h_item_pairs, sizeof(int4) * 2 * n_items,
                           cudaMemcpyHostToDevice, s)) ||
      (e = cudaMemcpyAsync(base + off_qinfo, h_qinfo, sizeof(int4) * n_queries,
                           cudaMemcpyHostToDevice, s)) ||
      (e = cudaMemcpyAsync(base + off_recs, h_recs, sizeof(int4) * 3 * n_units,
                           cudaMemcpyHostToDevice, s)) ||
      (n_merge > 0 && (e = cudaMemcpyAsync(base + off_merge, h_merge, sizeof(int32_t) * n_merge,
                                           cudaMemcpyHostToDevice, s))))
    return cuda_error(e, "kvc_decode_noalloc plan upload");

  DecodeArgs a = {};
  a.k_layer = static_cast<const uint8_t*>(d_k_layer);
  a.v_layer = static_cast<const uint8_t*>(d_v_layer);
  a.q = d_q;
  a.out = d_out;
  a.block_tables = d_block_tables;
  a.bt_stride = bt_stride;
  a.items = reinterpret_cast<const int4*>(base + off_items);
  a.qinfo = reinterpret_cast<const int4*>(base + off_qinfo);
  a.part_o = reinterpret_cast<float*>(base + off_part_o);
  a.part_ml = reinterpret_cast<float2*>(base + off_part_ml);
  a.counters = nullptr;  // not used by the tensor-core path
  a.sched_recs = reinterpret_cast<const int4*>(base + off_recs);
  a.n_units = n_units;
  a.sched_cap = n_units;
  a.queue = reinterpret_cast<unsigned*>(base + off_queue);
  a.n_sched_ctas = n_units > 0 ? n_ctas : 0;
  a.early_prefetch = 0;
  a.merge_queries = reinterpret_cast<const int32_t*>(base + off_merge);
  a.n_merge_queries = n_merge;
  a.merge_wph = merge_warps_per_head(max_splits);
  a.k_new = nullptr;
  a.v_new = nullptr;
  a.n_items = n_items;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.n_hchunk = nhc;
  a.head_dim = head_dim;
  a.page_size = page_size;
  a.num_pages = num_pages;
  a.scale_log2 = scale * kLog2e;
  if ((e = launch_decode(a, dtype, kLayoutCore, s)) != cudaSuccess)
    return cuda_error(e, "kvc_decode_noalloc kernels");
  return KVC_OK;
}
