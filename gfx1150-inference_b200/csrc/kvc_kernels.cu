// CUDA kernels of the B200 KV-cache decode path (sm_100a):
//   append_kernel      fused, vectorised scatter of new K/V rows into the paged pool
//   decode_mma_kernel  split-K flash-decoding GQA attention, 16-bit storage, tensor cores
//   decode_simt_kernel split-K GQA attention on CUDA cores (fp32 storage, odd head dims)
//   gather_kernel      pool -> token-major rows (bit-exact pool checks)
//   fill_normal_kernel seeded N(0, s^2) synthetic pool contents
//
// The attention computes, for every query m and q-head h, exactly the quantity of
// gfx1150-inference's gqa_online_softmax_kernel (src/kernels/attention.hip:35-123):
//   kv_h = h / (H / Hkv)                                   (attention.hip:59-60)
//   score_j = (q . k_j) * scale, scale used as given        (attention.hip:99)
//   out = sum_j softmax(score)_j * v_j over j < ctx        (attention.hip:75-113)
//   out = 0 when nothing is attended                       (attention.hip:115)
// with fp32 accumulation.  The work is organised the B200 way instead of one
// wave per (m, h) scanning every position: each CTA owns one KV head of one
// split of one query, streams that head's 16-position slabs once through shared
// memory with bulk copies, and serves all q-heads of the group from the same
// tile; splits are merged by the last CTA of a query to finish.
#include <stdio.h>

#include "kvc_device.cuh"
#include "kvc_internal.h"

namespace kvc {

// ---- device error word -----------------------------------------------------------
// [0] = first error code (KVC_DEVERR_*), [1] = auxiliary value.  One copy per
// device; read by the host after synchronising.
__device__ uint32_t g_kvc_deverr[2];

__device__ __forceinline__ void report_error(uint32_t code, uint32_t info) {
  if (atomicCAS(&g_kvc_deverr[0], 0u, code) == 0u) g_kvc_deverr[1] = info;
}

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
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
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
constexpr int kBarBytes = 128;

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
// Tensor-core split-K decode kernel (16-bit storage, head_dim multiple of 32).
//
// CTA = (split item, KV head, chunk of <= 8 q-heads); NW warps.  Warp w streams
// slabs w, w+NW, ... of the split through its own NS-deep ring of shared-memory
// stages (one bulk copy per K slab and per V slab, completion on an mbarrier).
// Per 16-position slab and warp:
//   S  = Q . K^T       mma m16n8k16: A = Q (rows = q-heads, zero-padded to 16),
//                      B = K^T fragments by ldmatrix from the core-matrix layout
//   online softmax on the S fragments (max over the 4 lanes of a row: 2 shuffles)
//   O^T += V^T . P^T   mma m16n8k16: A = V^T by ldmatrix.trans, B = P^T taken
//                      straight from the S accumulators (no shuffles)
// so K and V of a KV head are read from HBM exactly once for all its q-heads.
// =====================================================================================
template <typename T, int D, int NW, int NS>
__global__ void __launch_bounds__(NW * 32) decode_mma_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int SLAB_BYTES = kSlab * D * 2;     // one slab of K (or V)
  constexpr int STAGE_BYTES = 2 * SLAB_BYTES;   // K slab + V slab
  constexpr int KC = D / 16;                    // k-chunks of the QK product
  constexpr int MT = D / 16;                    // m-tiles of the PV product
  constexpr int U = D / 8;                      // 16-byte units per position

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;

  int b = blockIdx.x;
  const int hc = b % a.n_hchunk;
  b /= a.n_hchunk;
  const int kvh = b % a.num_kv_heads;
  b /= a.num_kv_heads;
  const int4 it = a.items[b];
  const int4 qi = a.qinfo[it.x];
  const int query = it.x, split = it.y, tb = it.z, te = it.w;
  const int hq0 = kvh * a.group + hc * 8;
  const int nh = min(8, a.group - hc * 8);
  const int ps = a.page_size;
  const int slabs_per_page = ps / kSlab;

  // Shared memory: [mbarriers (kBarBytes)] [NW x NS stages]; after the stream
  // loop the stage region is reused for the warp combine and the split merge.
  uint8_t* const region = smem + kBarBytes;
  uint8_t* stages = region + warp * NS * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * NS;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Q fragments: row gid of the A operand is q-head hq0 + gid (rows >= nh and the
  // upper 8 rows are zero).
  uint32_t qa[KC][2];
  {
    const T* qrow = reinterpret_cast<const T*>(a.q) +
                    (static_cast<size_t>(query) * a.num_heads + hq0 + gid) * D;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      if (gid < nh) {
        qa[kc][0] = *reinterpret_cast<const uint32_t*>(qrow + kc * 16 + 2 * tig);
        qa[kc][1] = *reinterpret_cast<const uint32_t*>(qrow + kc * 16 + 8 + 2 * tig);
      } else {
        qa[kc][0] = 0u;
        qa[kc][1] = 0u;
      }
    }
  }

  const int sb0 = tb / kSlab;
  const int sb1 = (te + kSlab - 1) / kSlab;
  const int nslabs = (sb1 - sb0 > warp) ? (sb1 - sb0 - warp + NW - 1) / NW : 0;
  const int32_t* bt_row = a.block_tables + static_cast<size_t>(qi.x) * a.bt_stride;
  const size_t head_off = static_cast<size_t>(kvh) * ps * D * 2;
  const size_t page_stride = static_cast<size_t>(a.num_kv_heads) * ps * D * 2;
  const uint64_t policy = l2_policy_evict_first();

  // Physical page of slab j, or -1 if the block table entry is out of range.
  auto slab_page = [&](int j) -> int {
    const int phys = bt_row[j / slabs_per_page];
    return (phys >= 0 && phys < a.num_pages) ? phys : -1;
  };
  auto issue = [&](int i) {  // lane 0 only
    const int j = sb0 + warp + i * NW;
    const int s = i % NS;
    const uint32_t bar = smem_u32(&bars[s]);
    const int phys = slab_page(j);
    if (phys < 0) {
      report_error(1u, static_cast<uint32_t>(bt_row[j / slabs_per_page]));
      mbar_arrive(bar);
      return;
    }
    const size_t off = static_cast<size_t>(phys) * page_stride + head_off +
                       static_cast<size_t>(j % slabs_per_page) * SLAB_BYTES;
    mbar_arrive_expect_tx(bar, STAGE_BYTES);
    const uint32_t dst = smem_u32(stages + s * STAGE_BYTES);
    bulk_g2s(dst, a.k_layer + off, SLAB_BYTES, bar, policy);
    bulk_g2s(dst + SLAB_BYTES, a.v_layer + off, SLAB_BYTES, bar, policy);
  };

  int issued = 0;
  if (lane == 0) {
    const int first = min(NS, nslabs);
    for (int i = 0; i < first; ++i) issue(i);
  }
  issued = min(NS, nslabs);
  __syncwarp();

  float m_run = kNegBig, l_run = 0.f;
  float o[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  int consumed = 0;
  for (int i = 0; i < nslabs; ++i) {
    const int s = i % NS;
    const uint32_t parity = static_cast<uint32_t>(i / NS) & 1u;
    const int j = sb0 + warp + i * NW;
    const bool ok = mbar_wait_bounded(smem_u32(&bars[s]), parity);
    if (__any_sync(0xffffffffu, !ok)) {
      if (lane == 0) report_error(2u /*KVC_DEVERR_WAIT_LIMIT*/, static_cast<uint32_t>(j));
      break;
    }
    consumed = i + 1;
    uint8_t* st = stages + s * STAGE_BYTES;
    const int valid = min(kSlab, te - j * kSlab);
    if (slab_page(j) >= 0) {
      if (valid < kSlab) {
        // Positions past the context may hold anything (the pool is not zeroed):
        // clear them so 0 * garbage never reaches the accumulators.
        const int nunits = (kSlab - valid) * U;
        for (int x = lane; x < 2 * nunits; x += 32) {
          const int kv = x / nunits, r = x - kv * nunits;
          const int t = valid + r / U, u = r - (r / U) * U;
          *reinterpret_cast<uint4*>(st + kv * SLAB_BYTES + unit_offset(kLayoutCore, t, u, U) * 16) =
              make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(st);
      const uint32_t vbase = kbase + SLAB_BYTES;

      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int k2 = 0; k2 < D / 32; ++k2) {
          uint32_t r0, r1, r2, r3;
          ldsm_x4(kbase + ((nt * U + k2 * 4 + (lane >> 3)) * 8 + (lane & 7)) * 16, r0, r1, r2, r3);
          Mma<T>::run(sc[nt], qa[2 * k2][0], 0u, qa[2 * k2][1], 0u, r0, r1);
          Mma<T>::run(sc[nt], qa[2 * k2 + 1][0], 0u, qa[2 * k2 + 1][1], 0u, r2, r3);
        }
      }
      // Lane (gid, tig) holds scores of q-head gid for positions 2tig, 2tig+1,
      // 8+2tig, 9+2tig of the slab.
      const int t0 = 2 * tig;
      const bool v0 = t0 < valid, v1 = t0 + 1 < valid, v2 = t0 + 8 < valid, v3 = t0 + 9 < valid;
      const float x0 = sc[0][0] * a.scale_log2, x1 = sc[0][1] * a.scale_log2;
      const float x2 = sc[1][0] * a.scale_log2, x3 = sc[1][1] * a.scale_log2;
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
      // Columns 2tig, 2tig+1 of O^T belong to q-heads 2tig, 2tig+1, whose alpha
      // lives in lanes (2tig)*4 and (2tig+1)*4.
      const float a_lo = __shfl_sync(0xffffffffu, alpha, (2 * tig) * 4);
      const float a_hi = __shfl_sync(0xffffffffu, alpha, (2 * tig + 1) * 4);
      const int jm = lane >> 3;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        o[mt][0] *= a_lo;
        o[mt][1] *= a_hi;
        o[mt][2] *= a_lo;
        o[mt][3] *= a_hi;
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vbase + (((jm >> 1) * U + 2 * mt + (jm & 1)) * 8 + (lane & 7)) * 16, r0, r1, r2, r3);
        Mma<T>::run(o[mt], r0, r1, r2, r3, pb0, pb1);
      }
    }
    __syncwarp();
    if (i + NS < nslabs) {
      if (lane == 0) {
        fence_proxy_async();
        issue(i + NS);
      }
      issued = i + NS + 1;
    }
  }
  // Error path only: wait (bounded) for copies still in flight into this warp's
  // stages before the shared memory is reused.
  for (int i = consumed; i < issued; ++i)
    (void)mbar_wait_bounded(smem_u32(&bars[i % NS]), static_cast<uint32_t>(i / NS) & 1u);

  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

  // ---- combine the NW warps of the CTA (stage memory is free now) ----
  __syncthreads();
  constexpr int OS = D + 4;
  float* wm = reinterpret_cast<float*>(region);   // [NW][8]
  float* wl = wm + NW * 8;                      // [NW][8]
  float* wo = wl + NW * 8;                      // [NW][8][OS]
  if (tig == 0) {
    wm[warp * 8 + gid] = m_run;
    wl[warp * 8 + gid] = l_run;
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    wo[(warp * 8 + 2 * tig) * OS + 16 * mt + gid] = o[mt][0];
    wo[(warp * 8 + 2 * tig + 1) * OS + 16 * mt + gid] = o[mt][1];
    wo[(warp * 8 + 2 * tig) * OS + 16 * mt + gid + 8] = o[mt][2];
    wo[(warp * 8 + 2 * tig + 1) * OS + 16 * mt + gid + 8] = o[mt][3];
  }
  __syncthreads();

  const int n_splits = qi.w;
  const int H = a.num_heads;
  for (int idx = threadIdx.x; idx < nh * D; idx += NW * 32) {
    const int h = idx / D, d = idx - (idx / D) * D;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w * 8 + h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = fast_exp2(wm[w * 8 + h] - M);
      L += wl[w * 8 + h] * f;
      O += wo[(w * 8 + h) * OS + d] * f;
    }
    if (n_splits == 1) {
      reinterpret_cast<T*>(a.out)[(static_cast<size_t>(query) * H + hq0 + h) * D + d] =
          from_f32<T>(L > 0.f ? O * (1.0f / L) : 0.f);
    } else {
      const size_t slot = static_cast<size_t>(qi.z + split) * H + hq0 + h;
      a.part_o[slot * D + d] = O;
      if (d == 0) a.part_ml[slot] = make_float2(M, L);
    }
  }
  if (n_splits > 1) {
    __syncthreads();  // the merge reuses the combine buffers
    finish_split<T>(a, reinterpret_cast<float*>(region), query, kvh, hc, qi.z, n_splits, hq0, nh);
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
  const int4 it = a.items[b];
  const int4 qi = a.qinfo[it.x];
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

  auto slab_page = [&](int j) -> int {
    const int phys = bt_row[j / slabs_per_page];
    return (phys >= 0 && phys < a.num_pages) ? phys : -1;
  };
  auto issue = [&](int i) {  // thread 0 only
    const int j = sb0 + i;
    const int s = i % NS;
    const uint32_t bar = smem_u32(&bars[s]);
    const int phys = slab_page(j);
    if (phys < 0) {
      report_error(1u, static_cast<uint32_t>(bt_row[j / slabs_per_page]));
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

constexpr int kNW = 4;

template <int D>
constexpr int mma_stages() {
  return D <= 128 ? 3 : 2;
}

template <typename T, int D>
cudaError_t run_mma(const DecodeArgs& a, cudaStream_t s) {
  constexpr int NS = mma_stages<D>();
  constexpr size_t stage_region = static_cast<size_t>(kNW) * NS * 2 * kSlab * D * 2;
  const size_t combine = (2 * kNW * 8 + static_cast<size_t>(kNW) * 8 * (D + 4)) * sizeof(float);
  const size_t merge = (8 * kMergeChunk + 8 * static_cast<size_t>(D) + 16) * sizeof(float);
  static_assert(kNW * NS * sizeof(uint64_t) <= kBarBytes, "mbarrier block too small");
  size_t smem = stage_region;
  if (combine > smem) smem = combine;
  if (merge > smem) smem = merge;
  smem += kBarBytes;
  auto kern = decode_mma_kernel<T, D, kNW, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(a.n_items) * a.num_kv_heads * a.n_hchunk;
  kern<<<grid, kNW * 32, smem, s>>>(a);
  return cudaGetLastError();
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
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
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
