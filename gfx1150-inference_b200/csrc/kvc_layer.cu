// Kernels of the layer pipeline (forward_layer_cached, attention.hip:603-695):
//
//   linear_kernel<WT, RT, MT>   y = x · Wᵀ for fp16 activations and GGML-quantized
//                               weights (F16, Q4_0, Q8_0, Q4_K, Q6_K), on the tensor
//                               cores (mma.sync m16n8k16, fp32 accumulate)
//   rmsnorm_kernel             RMSNorm, optionally fused with the residual add
//
// The reference's projections (dequantize.hip, matmul.hip) dequantize each weight to
// fp32 (d · (q − 8) etc.) and sum fp32 products.  Here the quantized integers go to
// the tensor cores exactly as fp16 (q − 8, q, q − 32 are small integers), the MMA
// sums q · x exactly in fp32 over each block, and the block's scale multiplies the
// block sum — the same per-block structure as the reference's kernels (block_sum
// then d · block_sum, dequantize.hip:120-137).  Q4_K's minimum term uses the block's
// Σx, from one more MMA against a matrix of ones.
//
// Decode rows are GEMV-shaped (m = tokens of one step, a handful), so the weights
// are the streamed operand: a CTA owns 16 · RT rows of W for 8 · MT tokens, its 8
// warps split k, and the partial sums are added in shared memory in warp order (the
// result does not depend on timing).  Every weight byte is read once per 8 · MT
// tokens; the unit loop keeps the next unit's loads in flight while it computes.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

#include "kvc_device.cuh"
#include "kvc_internal.h"

namespace kvc {
namespace {

constexpr int kLinWarps = 8;

// fp16x2 bit patterns of 1024 + b: the byte b of 0x64bb is the mantissa's low byte.
constexpr uint32_t kBias1024 = 0x64006400u;   // q           (Q4_K)
constexpr uint32_t kBias1032 = 0x64086408u;   // q − 8       (Q4_0)
constexpr uint32_t kBias1056 = 0x64206420u;   // q − 32      (Q6_K)
constexpr uint32_t kBias1152 = 0x64806480u;   // q (int8 ^ 0x80)   (Q8_0)
constexpr uint32_t kOnes = 0x3C003C00u;       // fp16x2 (1, 1)

// Four bytes b0..b3 of v → fp16x2 (b0, b1) − bias, (b2, b3) − bias: exact integers.
__device__ __forceinline__ void bytes_to_h2(uint32_t v, uint32_t bias, uint32_t& lo,
                                            uint32_t& hi) {
  const uint32_t l = __byte_perm(v, 0x64646464u, 0x4140u);
  const uint32_t h = __byte_perm(v, 0x64646464u, 0x4342u);
  asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(l), "r"(bias));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(h), "r"(bias));
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}
// Four bytes at a 2-byte aligned address.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) {
  return ld_u16(p) | (ld_u16(p + 2) << 16);
}
__device__ __forceinline__ float h_bits_to_f32(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// 6-bit scale and min of 32-weight group j of a Q4_K super-block (GGML's packing of
// scales[12] as three words s0, s1, s2; gguf_parser.py:490-495).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j,
                                              int& sc, int& mn) {
  if (j < 4) {
    sc = (s0 >> (8 * j)) & 63;
    mn = (s1 >> (8 * j)) & 63;
  } else {
    const int jj = j - 4;
    sc = ((s2 >> (8 * jj)) & 0x0F) | (((s0 >> (8 * jj + 6)) & 3) << 4);
    mn = ((s2 >> (8 * jj + 4)) & 0x0F) | (((s1 >> (8 * jj + 6)) & 3) << 4);
  }
}

template <int WT>
struct WTraits;
// unit: the k-range one warp takes at a time (a block, or a super-block's quarter)
template <>
struct WTraits<kWF16> {
  static constexpr int kUnitK = 32;
};
template <>
struct WTraits<kWQ4_0> {
  static constexpr int kUnitK = 32;   // one 18-byte block
};
template <>
struct WTraits<kWQ8_0> {
  static constexpr int kUnitK = 32;   // one 34-byte block
};
template <>
struct WTraits<kWQ4_K> {
  static constexpr int kUnitK = 64;   // a quarter of a 144-byte super-block
};
template <>
struct WTraits<kWQ6_K> {
  static constexpr int kUnitK = 64;   // a quarter of a 210-byte super-block
};

// Raw words of one unit for this thread: per row tile and row half (gid, gid + 8)
// up to six 32-bit words of weights and scales.
template <int RT>
struct Raw {
  uint32_t w[RT][2][6];
};

template <int WT, int RT>
__device__ __forceinline__ void load_unit(Raw<RT>& r, const uint8_t* const (&wr)[RT][2], int u,
                                          int tig) {
#pragma unroll
  for (int t = 0; t < RT; ++t)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint8_t* row = wr[t][h];
      if (row == nullptr) {
#pragma unroll
        for (int i = 0; i < 6; ++i) r.w[t][h][i] = 0u;
        continue;
      }
      if constexpr (WT == kWF16) {
        // weights 4tig .. 4tig + 3 of chunk 0 (words 0, 1) and of chunk 1 (words 2, 3)
        const uint2 a = *reinterpret_cast<const uint2*>(row + static_cast<size_t>(u) * 64 + 8 * tig);
        const uint2 b =
            *reinterpret_cast<const uint2*>(row + static_cast<size_t>(u) * 64 + 32 + 8 * tig);
        r.w[t][h][0] = a.x;
        r.w[t][h][1] = a.y;
        r.w[t][h][2] = b.x;
        r.w[t][h][3] = b.y;
      } else if constexpr (WT == kWQ4_0) {
        const uint8_t* blk = row + static_cast<size_t>(u) * 18;
        r.w[t][h][0] = ld_u16(blk);                    // d
        r.w[t][h][1] = ld_u32_a2(blk + 2 + 4 * tig);    // qs[4tig .. 4tig + 3]
      } else if constexpr (WT == kWQ8_0) {
        const uint8_t* blk = row + static_cast<size_t>(u) * 34;
        r.w[t][h][0] = ld_u16(blk);
        r.w[t][h][1] = ld_u32_a2(blk + 2 + 4 * tig);        // weights 4tig.. of chunk 0
        r.w[t][h][2] = ld_u32_a2(blk + 2 + 16 + 4 * tig);   // weights 16 + 4tig..
      } else if constexpr (WT == kWQ4_K) {
        const int sb = u >> 2, st = u & 3;   // quarter st: groups 2st (low) and 2st + 1 (high)
        const uint8_t* blk = row + static_cast<size_t>(sb) * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);   // d, dmin, scales[12]
        r.w[t][h][0] = hdr.x;
        r.w[t][h][1] = hdr.y;
        r.w[t][h][2] = hdr.z;
        r.w[t][h][3] = hdr.w;
        r.w[t][h][4] = *reinterpret_cast<const uint32_t*>(blk + 16 + 32 * st + 4 * tig);
        r.w[t][h][5] = *reinterpret_cast<const uint32_t*>(blk + 16 + 32 * st + 16 + 4 * tig);
      } else {  // kWQ6_K: quarter (n, s) = (u >> 1 & 1, u & 1) of super-block u >> 2
        const int sb = u >> 2, n = (u >> 1) & 1, s = u & 1;
        const uint8_t* blk = row + static_cast<size_t>(sb) * 210;
        r.w[t][h][0] = ld_u32_a2(blk + 64 * n + 16 * s + 4 * tig);        // quarters t = 0, 2
        r.w[t][h][1] = ld_u32_a2(blk + 64 * n + 32 + 16 * s + 4 * tig);   // quarters t = 1, 3
        r.w[t][h][2] = ld_u32_a2(blk + 128 + 32 * n + 16 * s + 4 * tig);  // high bits
        // scales of the four 16-weight groups 8n + 2t + s (bytes 192 + 8n + 2t + s)
        r.w[t][h][3] = ld_u32_a2(blk + 192 + 8 * n);       // t = 0, 1
        r.w[t][h][4] = ld_u32_a2(blk + 192 + 8 * n + 4);   // t = 2, 3
        r.w[t][h][5] = ld_u16(blk + 208);                  // d
      }
    }
}

// First error of a kernel: KVC_DEVERR_WAIT_LIMIT with the stage it gave up on.
__device__ __forceinline__ void report_lin_error(const LinearArgs& a, uint32_t info) {
  if (a.err != nullptr && atomicCAS(a.err, 0u, 2u /*KVC_DEVERR_WAIT_LIMIT*/) == 0u) a.err[1] = info;
}

// 16-weight chunks of a unit and the k offset of chunk c within it.
template <int WT>
constexpr int kChunks = (WT == kWQ4_K || WT == kWQ6_K) ? 4 : 2;
template <int WT>
__host__ __device__ constexpr int chunk_k(int c) {
  return (WT == kWQ6_K ? 32 : 16) * c;
}

// B fragments of the 16-weight chunk at k0 for the token tiles (the k order
// 4tig .. 4tig + 3 of the A fragments); rows past m read as zero.
template <int MT>
struct BFrag {
  const __half* row[MT];   // token rows (global or shared), null past m
  int tig;
  __device__ __forceinline__ void operator()(int k0, uint32_t (&b)[MT][2]) const {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      if (row[mt] != nullptr) {
        const uint2 v = *reinterpret_cast<const uint2*>(row[mt] + k0 + 4 * tig);
        b[mt][0] = v.x;
        b[mt][1] = v.y;
      } else {
        b[mt][0] = b[mt][1] = 0u;
      }
    }
  }
  // every chunk of the unit whose first weight sits at k0
  template <int WT>
  __device__ __forceinline__ void unit(int k0, uint32_t (&bf)[kChunks<WT>][MT][2]) const {
#pragma unroll
    for (int c = 0; c < kChunks<WT>; ++c) (*this)(k0 + chunk_k<WT>(c), bf[c]);
  }
};

// acc += this thread's share of unit u (k range [u·UK, (u + 1)·UK)) of the CTA's
// rows times the tokens; `cur` holds the unit's raw weight words, bf its B
// fragments (chunk c at k offset chunk_k<WT>(c) of the unit).
template <int WT, int RT, int MT>
__device__ __forceinline__ void compute_unit(const Raw<RT>& cur, int u,
                                             const uint32_t (&bf)[kChunks<WT>][MT][2],
                                             float (&acc)[RT][MT][4]) {
  if constexpr (WT == kWF16) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
      for (int t = 0; t < RT; ++t)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          Mma<__half>::run(acc[t][mt], cur.w[t][0][2 * c], cur.w[t][1][2 * c],
                           cur.w[t][0][2 * c + 1], cur.w[t][1][2 * c + 1], bf[c][mt][0],
                           bf[c][mt][1]);
    }
  } else if constexpr (WT == kWQ4_0 || WT == kWQ8_0) {
    float tmp[RT][MT][4];
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) tmp[t][mt][0] = tmp[t][mt][1] = tmp[t][mt][2] = tmp[t][mt][3] = 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
      for (int t = 0; t < RT; ++t) {
        uint32_t lo[2], hi[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if constexpr (WT == kWQ4_0) {
            const uint32_t q = c == 0 ? (cur.w[t][h][1] & 0x0F0F0F0Fu)
                                      : ((cur.w[t][h][1] >> 4) & 0x0F0F0F0Fu);
            bytes_to_h2(q, kBias1032, lo[h], hi[h]);
          } else {
            bytes_to_h2(cur.w[t][h][1 + c] ^ 0x80808080u, kBias1152, lo[h], hi[h]);
          }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          Mma<__half>::run(tmp[t][mt], lo[0], lo[1], hi[0], hi[1], bf[c][mt][0], bf[c][mt][1]);
      }
    }
#pragma unroll
    for (int t = 0; t < RT; ++t) {
      const float d0 = h_bits_to_f32(cur.w[t][0][0]), d1 = h_bits_to_f32(cur.w[t][1][0]);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        acc[t][mt][0] += d0 * tmp[t][mt][0];
        acc[t][mt][1] += d0 * tmp[t][mt][1];
        acc[t][mt][2] += d1 * tmp[t][mt][2];
        acc[t][mt][3] += d1 * tmp[t][mt][3];
      }
    }
  } else if constexpr (WT == kWQ4_K) {
    const int st = u & 3;
#pragma unroll
    for (int g = 0; g < 2; ++g) {  // group j = 2st + g: low (g = 0) or high nibbles
      const int j = 2 * st + g;
      float tmp[RT][MT][4], sx[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        sx[mt][0] = sx[mt][1] = sx[mt][2] = sx[mt][3] = 0.f;
#pragma unroll
        for (int t = 0; t < RT; ++t) tmp[t][mt][0] = tmp[t][mt][1] = tmp[t][mt][2] = tmp[t][mt][3] = 0.f;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t (&b)[MT][2] = bf[2 * g + c];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          Mma<__half>::run(sx[mt], kOnes, kOnes, kOnes, kOnes, b[mt][0], b[mt][1]);
#pragma unroll
        for (int t = 0; t < RT; ++t) {
          uint32_t lo[2], hi[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t q = (cur.w[t][h][4 + c] >> (4 * g)) & 0x0F0F0F0Fu;
            bytes_to_h2(q, kBias1024, lo[h], hi[h]);
          }
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            Mma<__half>::run(tmp[t][mt], lo[0], lo[1], hi[0], hi[1], b[mt][0], b[mt][1]);
        }
      }
#pragma unroll
      for (int t = 0; t < RT; ++t) {
        float ds[2], dm[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int sc, mn;
          q4k_scale_min(cur.w[t][h][1], cur.w[t][h][2], cur.w[t][h][3], j, sc, mn);
          ds[h] = h_bits_to_f32(cur.w[t][h][0] & 0xFFFFu) * static_cast<float>(sc);
          dm[h] = h_bits_to_f32(cur.w[t][h][0] >> 16) * static_cast<float>(mn);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[t][mt][0] += ds[0] * tmp[t][mt][0] - dm[0] * sx[mt][0];
          acc[t][mt][1] += ds[0] * tmp[t][mt][1] - dm[0] * sx[mt][1];
          acc[t][mt][2] += ds[1] * tmp[t][mt][2] - dm[1] * sx[mt][2];
          acc[t][mt][3] += ds[1] * tmp[t][mt][3] - dm[1] * sx[mt][3];
        }
      }
    }
  } else {  // kWQ6_K: quarter (n, s) of a super-block, four 16-weight groups
    const int s6 = u & 1;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {  // group t: weights 128n + 32t + 16s ..
      const uint32_t (&b)[MT][2] = bf[q4];
#pragma unroll
      for (int t = 0; t < RT; ++t) {
        float tmp[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) tmp[mt][0] = tmp[mt][1] = tmp[mt][2] = tmp[mt][3] = 0.f;
        uint32_t lo[2], hi[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t nib = ((cur.w[t][h][q4 & 1] >> (4 * (q4 >> 1))) & 0x0F0F0F0Fu);
          const uint32_t top = ((cur.w[t][h][2] >> (2 * q4)) & 0x03030303u) << 4;
          bytes_to_h2(nib | top, kBias1056, lo[h], hi[h]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          Mma<__half>::run(tmp[mt], lo[0], lo[1], hi[0], hi[1], b[mt][0], b[mt][1]);
        float ds[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          // scale byte 8n + 2q4 + s: word 3 holds bytes 0..3 (q4 = 0, 1), word 4 bytes 4..7
          const uint32_t word = q4 < 2 ? cur.w[t][h][3] : cur.w[t][h][4];
          const int byte = 2 * (q4 & 1) + s6;
          const int sc = static_cast<int>(static_cast<int8_t>((word >> (8 * byte)) & 0xFFu));
          ds[h] = h_bits_to_f32(cur.w[t][h][5]) * static_cast<float>(sc);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[t][mt][0] += ds[0] * tmp[mt][0];
          acc[t][mt][1] += ds[0] * tmp[mt][1];
          acc[t][mt][2] += ds[1] * tmp[mt][2];
          acc[t][mt][3] += ds[1] * tmp[mt][3];
        }
      }
    }
  }
}

// k of the first weight of unit u as the B loader sees it (Q6_K units are
// (half, s) quarters: their groups start at 128·half + 16·s, 32 apart).
template <int WT>
__device__ __forceinline__ int unit_k0(int u) {
  if constexpr (WT == kWQ6_K) return (u >> 2) * 256 + 128 * ((u >> 1) & 1) + 16 * (u & 1);
  else if constexpr (WT == kWQ4_K) return (u >> 2) * 256 + 64 * (u & 3);
  else return u * 32;
}

// The CTA's place: segment s, first row n0 (of each half for SwiGLU), first token m0.
struct CtaPlace {
  int s, n0, m0;
};
template <int RT, int MT>
__device__ __forceinline__ CtaPlace cta_place(const LinearArgs& a) {
  CtaPlace p;
  p.s = 0;
  if (a.epi == kEpiSwiglu) {
    p.n0 = blockIdx.x * (RT * 8);
  } else {
    while (p.s + 1 < a.n_seg && static_cast<int>(blockIdx.x) >= a.seg_cta0[p.s + 1]) ++p.s;
    p.n0 = (blockIdx.x - a.seg_cta0[p.s]) * RT * 16;
  }
  p.m0 = blockIdx.y * MT * 8;
  return p;
}
// First row of tile t in its segment, and the segment.
template <int RT>
__device__ __forceinline__ int tile_row(const LinearArgs& a, const CtaPlace& p, int t, int& sg) {
  if (a.epi == kEpiSwiglu) {
    constexpr int P = RT / 2 > 0 ? RT / 2 : 1;
    sg = t < P ? 0 : 1;
    return p.n0 + 16 * (t % P);
  }
  sg = p.s;
  return p.n0 + 16 * t;
}

// Sum of the warps' partial tiles in warp order, epilogue, store.
template <int RT, int MT>
__device__ __forceinline__ void reduce_store(const LinearArgs& a, const CtaPlace& p,
                                             float (*red)[MT * 8][RT * 16 + 1],
                                             const float (&acc)[RT][MT][4], int warp, int gid,
                                             int tig) {
  constexpr int R = RT * 16, TOK = MT * 8;
#pragma unroll
  for (int t = 0; t < RT; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[warp][mt * 8 + 2 * tig + (e & 1)][t * 16 + gid + (e >= 2 ? 8 : 0)] = acc[t][mt][e];
  __syncthreads();
  if (a.epi != kEpiSwiglu) {
    const LinearSeg& sg = a.seg[p.s];
    for (int e = threadIdx.x; e < TOK * R; e += blockDim.x) {
      const int tok = e / R, r = e - (e / R) * R;
      const int m = p.m0 + tok, n = p.n0 + r;
      if (m >= a.m || n >= sg.n) continue;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kLinWarps; ++w) v += red[w][tok][r];
      __half y = __float2half_rn(v);
      const size_t o = static_cast<size_t>(m) * sg.out_ld + n;
      if (a.epi == kEpiResidual) y = __float2half_rn(__half2float(a.res[o]) + __half2float(y));
      sg.out[o] = y;
    }
  } else {
    constexpr int RH = R / 2;
    const LinearSeg& sg = a.seg[0];
    for (int e = threadIdx.x; e < TOK * RH; e += blockDim.x) {
      const int tok = e / RH, r = e - (e / RH) * RH;
      const int m = p.m0 + tok, n = p.n0 + r;
      if (m >= a.m || n >= sg.n) continue;
      float vg = 0.f, vu = 0.f;
#pragma unroll
      for (int w = 0; w < kLinWarps; ++w) {
        vg += red[w][tok][r];
        vu += red[w][tok][r + RH];
      }
      const float g = __half2float(__float2half_rn(vg));
      const float up = __half2float(__float2half_rn(vu));
      sg.out[static_cast<size_t>(m) * sg.out_ld + n] = __float2half_rn(g / (1.0f + expf(-g)) * up);
    }
  }
}

// Units in flight per warp of the register-pipelined kernel: deep enough that a
// warp keeps about 2 KB of weight rows (and their B fragments) in flight.
template <int WT, int RT, int MT>
__host__ __device__ constexpr int pipe_depth() {
  if constexpr (MT > 1) return 2;
  if constexpr (WT == kWQ4_K || WT == kWQ6_K) return RT == 1 ? 4 : 2;
  return RT == 1 ? 8 : (RT == 2 ? 4 : 2);
}

// Each warp takes units warp, warp + 8, ... of the CTA's rows and keeps the next
// pipe_depth units' weight words and B fragments in registers, loaded straight
// from global memory: every load is issued that many units before its use.
template <int WT, int RT, int MT>
__global__ void __launch_bounds__(256) linear_kernel(const LinearArgs a) {
  constexpr int UK = WTraits<WT>::kUnitK;
  constexpr int DEPTH = pipe_depth<WT, RT, MT>();
  __shared__ float red[kLinWarps][MT * 8][RT * 16 + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const CtaPlace p = cta_place<RT, MT>(a);
  const uint8_t* wr[RT][2];
#pragma unroll
  for (int t = 0; t < RT; ++t) {
    int sg;
    const int row = tile_row<RT>(a, p, t, sg);
    const bool ok = row < a.seg[sg].n;
    wr[t][0] = ok ? a.seg[sg].w + static_cast<size_t>(row + gid) * a.row_bytes : nullptr;
    wr[t][1] = ok ? a.seg[sg].w + static_cast<size_t>(row + gid + 8) * a.row_bytes : nullptr;
  }
  BFrag<MT> load_b;
  load_b.tig = tig;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int m = p.m0 + mt * 8 + gid;
    load_b.row[mt] = m < a.m ? a.x + static_cast<size_t>(m) * a.x_ld : nullptr;
  }
  float acc[RT][MT][4];
#pragma unroll
  for (int t = 0; t < RT; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[t][mt][0] = acc[t][mt][1] = acc[t][mt][2] = acc[t][mt][3] = 0.f;
  const int n_units = a.k / UK;
  const int mine = n_units > warp ? (n_units - warp + kLinWarps - 1) / kLinWarps : 0;
  Raw<RT> ring[DEPTH];
  uint32_t ring_b[DEPTH][kChunks<WT>][MT][2];
#pragma unroll
  for (int j = 0; j < DEPTH; ++j)
    if (j < mine) {
      const int u = warp + kLinWarps * j;
      load_unit<WT, RT>(ring[j], wr, u, tig);
      load_b.template unit<WT>(unit_k0<WT>(u), ring_b[j]);
    }
#pragma unroll 1
  for (int base = 0; base < mine; base += DEPTH) {
#pragma unroll
    for (int j = 0; j < DEPTH; ++j) {
      const int i = base + j;
      if (i < mine) {
        compute_unit<WT, RT, MT>(ring[j], warp + kLinWarps * i, ring_b[j], acc);
        if (i + DEPTH < mine) {
          const int u = warp + kLinWarps * (i + DEPTH);
          load_unit<WT, RT>(ring[j], wr, u, tig);
          load_b.template unit<WT>(unit_k0<WT>(u), ring_b[j]);
        }
      }
    }
  }
  reduce_store<RT, MT>(a, p, red, acc, warp, gid, tig);
}

// Weights (k) per stage of the staged kernel: whole blocks, a multiple of 16
// bytes per row, and 1-2 KB per row so each bulk copy is long.
__host__ __device__ constexpr int stage_k(int w_type) {
  return (w_type == kWQ8_0 || w_type == kWF16) ? 1024 : 2048;
}

// Staged variant: the CTA's weight rows and token rows stream through a ring of
// a.stages shared-memory stages, each a k-range of a.stage_k weights, filled by
// bulk copies (the TMA engine; one copy per row segment, issued by the lanes of
// warp 0) that complete on the stage's mbarrier.  The 8 warps each take one unit
// (four for Q6_K) of a stage; after all of them are done with it, the stage is
// refilled with the range a.stages ahead, so that many ranges of every row are in
// flight.  Waits are bounded; a wait that runs out reports KVC_DEVERR_WAIT_LIMIT,
// waits (bounded) for the copies still in flight and returns without output.
template <int WT, int RT, int MT>
__global__ void __launch_bounds__(256) linear_tma_kernel(const LinearArgs a) {
  constexpr int R = RT * 16, TOK = MT * 8;
  constexpr int UK = WTraits<WT>::kUnitK;
  constexpr int SK = stage_k(WT);             // weights (k) per stage
  constexpr int US = SK / UK;                 // units per stage
  constexpr int kLinBatch = (RT == 1 && (WT == kWQ4_0 || WT == kWQ8_0)) ? 4 : 2;
  static_assert((US / kLinWarps) % kLinBatch == 0, "units per warp and stage");
  constexpr uint32_t XRS = SK * 2 + 16;       // shared-memory stride of a token row
  __shared__ float red[kLinWarps][TOK][R + 1];
  __shared__ __align__(8) uint64_t full[kMaxLinStages];
  extern __shared__ __align__(128) uint8_t ring[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const CtaPlace p = cta_place<RT, MT>(a);
  const int NS = a.stages;
  const uint32_t SBR = a.stage_row_bytes;                 // weight bytes per row per stage
  const uint32_t WRS = SBR + 16;   // shared-memory stride of a weight row (spreads the banks)
  const size_t stage_bytes = static_cast<size_t>(R) * WRS + static_cast<size_t>(a.stage_tok) * XRS;
  // rows and tokens of this CTA
  const uint8_t* tile_w[RT];
  int valid_rows = 0;
#pragma unroll
  for (int t = 0; t < RT; ++t) {
    int sg;
    const int row = tile_row<RT>(a, p, t, sg);
    tile_w[t] = row < a.seg[sg].n ? a.seg[sg].w + static_cast<size_t>(row) * a.row_bytes : nullptr;
    valid_rows += tile_w[t] != nullptr ? 16 : 0;
  }
  const int valid_tok = min(TOK, a.m - p.m0);
  const uint32_t tx = static_cast<uint32_t>(valid_rows) * SBR + static_cast<uint32_t>(valid_tok) * SK * 2;
  const int n_stages = a.k / SK;
  const uint64_t policy = l2_policy_evict_first();
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(smem_u32(&full[i]), 1);
    fence_mbar_init();
  }
  __syncthreads();
  // warp 0: lane 0 arms the barrier, then the lanes copy one row segment each
  auto issue = [&](int st) {
    const int slot = st % NS;
    uint8_t* buf = ring + slot * stage_bytes;
    const uint32_t bar = smem_u32(&full[slot]);
    if (lane == 0) mbar_arrive_expect_tx(bar, tx);
    __syncwarp();
    for (int i = lane; i < R + valid_tok; i += 32) {
      if (i < R) {
        const uint8_t* tw = tile_w[i >> 4];
        if (tw != nullptr)
          bulk_g2s(smem_u32(buf + static_cast<size_t>(i) * WRS),
                   tw + static_cast<size_t>(i & 15) * a.row_bytes + static_cast<size_t>(st) * SBR,
                   SBR, bar, policy);
      } else {
        const int tk = i - R;
        bulk_g2s(smem_u32(buf + static_cast<size_t>(R) * WRS + static_cast<size_t>(tk) * XRS),
                 a.x + static_cast<size_t>(p.m0 + tk) * a.x_ld + static_cast<size_t>(st) * SK,
                 SK * 2, bar, policy);
      }
    }
  };
  if (warp == 0)
    for (int st = 0; st < min(NS, n_stages); ++st) issue(st);
  float acc[RT][MT][4];
#pragma unroll
  for (int t = 0; t < RT; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[t][mt][0] = acc[t][mt][1] = acc[t][mt][2] = acc[t][mt][3] = 0.f;
  int done = 0;   // stages consumed
  bool dead = false;
#pragma unroll 1
  for (int st = 0; st < n_stages; ++st) {
    const int slot = st % NS;
    const bool ok = mbar_wait_bounded(smem_u32(&full[slot]), static_cast<uint32_t>(st / NS) & 1u);
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) report_lin_error(a, static_cast<uint32_t>(st));
      dead = true;
      break;
    }
    // Shared-memory rows of the stage.  Tiles past n and token rows past m hold no
    // copy: they are read anyway (within the stage) and their results never stored,
    // so every pointer stays a plain shared-memory pointer.
    const uint8_t* buf = ring + slot * stage_bytes;
    const uint8_t* wr[RT][2];
#pragma unroll
    for (int t = 0; t < RT; ++t) {
      wr[t][0] = buf + static_cast<size_t>(t * 16 + gid) * WRS;
      wr[t][1] = buf + static_cast<size_t>(t * 16 + gid + 8) * WRS;
    }
    BFrag<MT> load_b;
    load_b.tig = tig;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int tk = min(mt * 8 + gid, valid_tok - 1);
      load_b.row[mt] = reinterpret_cast<const __half*>(buf + static_cast<size_t>(R) * WRS +
                                                       static_cast<size_t>(tk) * XRS);
    }
    // this warp's units of the stage, loads first (all of them are independent)
    constexpr int UPW = US / kLinWarps;
#pragma unroll
    for (int i0 = 0; i0 < UPW; i0 += kLinBatch) {
      Raw<RT> cur[kLinBatch];
      uint32_t bf[kLinBatch][kChunks<WT>][MT][2];
#pragma unroll
      for (int i = 0; i < kLinBatch; ++i) {
        const int ul = warp + kLinWarps * (i0 + i);
        load_unit<WT, RT>(cur[i], wr, ul, tig);
        load_b.template unit<WT>(unit_k0<WT>(ul), bf[i]);
      }
#pragma unroll
      for (int i = 0; i < kLinBatch; ++i)
        compute_unit<WT, RT, MT>(cur[i], warp + kLinWarps * (i0 + i), bf[i], acc);
    }
    done = st + 1;
    __syncthreads();   // every warp is done with the stage
    if (warp == 0 && st + NS < n_stages) issue(st + NS);
  }
  if (dead) {
    // copies still in flight land before the CTA exits
    if (threadIdx.x == 0)
      for (int st = done; st < min(n_stages, done + NS); ++st)
        (void)mbar_wait_bounded(smem_u32(&full[st % NS]), static_cast<uint32_t>(st / NS) & 1u);
    return;
  }
  reduce_store<RT, MT>(a, p, red, acc, warp, gid, tig);
}

// One CTA per row: fp32 sum of squares, then x / sqrt(mean + eps) · w.  Rows of up
// to 256 · 8 · kNormVec elements are held in registers (16-byte loads, one read
// of x, res and w each); longer rows take the element loop.
constexpr int kNormVec = 8;
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __half* __restrict__ x,
                                                      const __half* __restrict__ res,
                                                      const __half* __restrict__ w,
                                                      __half* __restrict__ h_out,
                                                      __half* __restrict__ out, int k,
                                                      float eps) {
  __shared__ float part[8];
  const size_t row = static_cast<size_t>(blockIdx.x) * k;
  const bool vec = k % 8 == 0 && k <= 256 * 8 * kNormVec &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                     reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(res) |
                     reinterpret_cast<uintptr_t>(h_out)) & 15u) == 0;
  auto block_sum = [&](float ss) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += part[i];
    return tot;
  };
  if (vec) {
    const int n8 = k / 8;
    uint4 v[kNormVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
      const int c = threadIdx.x + 256 * j;
      if (c < n8) {
        v[j] = reinterpret_cast<const uint4*>(x + row)[c];
        if (res != nullptr) {
          const uint4 r = reinterpret_cast<const uint4*>(res + row)[c];
          __half2* hv = reinterpret_cast<__half2*>(&v[j]);
          const __half2* hr = reinterpret_cast<const __half2*>(&r);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 a = __half22float2(hv[e]), b = __half22float2(hr[e]);
            hv[e] = __floats2half2_rn(a.x + b.x, a.y + b.y);
          }
          reinterpret_cast<uint4*>(h_out + row)[c] = v[j];
        }
        const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = __half22float2(hv[e]);
          ss += a.x * a.x + a.y * a.y;
        }
      }
    }
    const float rms = sqrtf(block_sum(ss) / static_cast<float>(k) + eps);
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
      const int c = threadIdx.x + 256 * j;
      if (c < n8) {
        const uint4 wv = reinterpret_cast<const uint4*>(w)[c];
        const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
        const __half2* hw = reinterpret_cast<const __half2*>(&wv);
        uint4 o;
        __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = __half22float2(hv[e]), b = __half22float2(hw[e]);
          ho[e] = __floats2half2_rn(a.x / rms * b.x, a.y / rms * b.y);
        }
        reinterpret_cast<uint4*>(out + row)[c] = o;
      }
    }
    return;
  }
  const __half* xr = x + row;
  float ss = 0.f;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    float v = __half2float(xr[i]);
    if (res != nullptr) {
      const __half h = __float2half_rn(v + __half2float(res[row + i]));
      h_out[row + i] = h;
      v = __half2float(h);
    }
    ss += v * v;
  }
  const float rms = sqrtf(block_sum(ss) / static_cast<float>(k) + eps);
  const __half* src = res != nullptr ? h_out + row : xr;
  for (int i = threadIdx.x; i < k; i += blockDim.x)
    out[row + i] = __float2half_rn(__half2float(src[i]) / rms * __half2float(w[i]));
}

// SwiGLU of two fp16 arrays (mlp.hip:18-31), for gate and up of different types.
__global__ void __launch_bounds__(256) swiglu_kernel(const __half* __restrict__ gate,
                                                     const __half* __restrict__ up,
                                                     __half* __restrict__ out, size_t n) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float g = __half2float(gate[i]);
    out[i] = __float2half_rn(g / (1.0f + expf(-g)) * __half2float(up[i]));
  }
}

template <auto Kernel>
cudaError_t smem_opt_in(size_t bytes) {
  static std::atomic<size_t> done[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
  if (e == cudaSuccess && dev >= 0 && dev < 64) {
    size_t cur = done[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !done[dev].compare_exchange_weak(cur, bytes)) {
    }
  }
  return e;
}

template <int WT, int RT, int MT>
cudaError_t run_linear(const LinearArgs& a, int n_ctas, bool staged, size_t ring_bytes,
                       cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(n_ctas),
                  static_cast<unsigned>((a.m + MT * 8 - 1) / (MT * 8)), 1);
  if (staged) {
    cudaError_t e = smem_opt_in<linear_tma_kernel<WT, RT, MT>>(ring_bytes);
    if (e != cudaSuccess) return e;
    linear_tma_kernel<WT, RT, MT><<<grid, 32 * kLinWarps, ring_bytes, s>>>(a);
  } else {
    linear_kernel<WT, RT, MT><<<grid, 32 * kLinWarps, 0, s>>>(a);
  }
  return cudaGetLastError();
}

template <int WT>
cudaError_t run_linear_t(LinearArgs& a, int rt, int mt, int n_ctas, cudaStream_t s) {
  // The staged kernel takes rows that are whole multiples of 16 bytes, k a whole
  // number of stages and 16-byte aligned operands (every Llama-family shape).
  constexpr int SK = stage_k(WT);
  int per = 0, bytes = 0;
  weight_block(WT, &per, &bytes);
  bool staged = a.row_bytes % 16 == 0 && a.k % SK == 0 &&
                (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && (a.x_ld * 2) % 16 == 0;
  for (int i = 0; i < a.n_seg; ++i)
    staged = staged && (reinterpret_cast<uintptr_t>(a.seg[i].w) & 15u) == 0;
  const uint32_t sbr = static_cast<uint32_t>(SK / per * bytes);
  const int tok_rows = std::min(mt * 8, a.m);   // token rows of x per stage
  const size_t stage_bytes = static_cast<size_t>(rt * 16) * (sbr + 16) +
                             static_cast<size_t>(tok_rows) * (SK * 2 + 16);
  // about 96 KB of ring per CTA (two CTAs per SM), at least two stages
  int ns = static_cast<int>(std::min<size_t>(kMaxLinStages, (96u << 10) / stage_bytes));
  if (ns < 2) {
    ns = 2;
    staged = staged && stage_bytes * 2 <= (160u << 10);
  }
  a.stages = ns;
  a.stage_row_bytes = sbr;
  a.stage_tok = tok_rows;
  const size_t ring = static_cast<size_t>(ns) * stage_bytes;
  if (mt == 1) {
    if (rt == 1) return run_linear<WT, 1, 1>(a, n_ctas, staged, ring, s);
    if (rt == 2) return run_linear<WT, 2, 1>(a, n_ctas, staged, ring, s);
    return run_linear<WT, 4, 1>(a, n_ctas, staged, ring, s);
  }
  if (rt == 1) return run_linear<WT, 1, 4>(a, n_ctas, staged, ring, s);
  return run_linear<WT, 2, 4>(a, n_ctas, staged, ring, s);
}

}  // namespace

void weight_block(int w_type, int* per, int* bytes) {
  switch (w_type) {
    case kWF16: *per = 1; *bytes = 2; return;
    case kWQ4_0: *per = 32; *bytes = 18; return;
    case kWQ8_0: *per = 32; *bytes = 34; return;
    case kWQ4_K: *per = 256; *bytes = 144; return;
    case kWQ6_K: *per = 256; *bytes = 210; return;
    default: *per = 0; *bytes = 0; return;
  }
}

cudaError_t launch_linear(LinearArgs& a, cudaStream_t s) {
  if (a.m <= 0) return cudaSuccess;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;
  }
  const int mt = a.m <= 8 ? 1 : 4;
  int rows = 0;
  for (int i = 0; i < a.n_seg; ++i) rows += a.seg[i].n;
  // Row tiles per CTA: more rows per CTA (fewer re-reads of x) while the grid still
  // has about two CTAs per SM; a SwiGLU CTA pairs gate and up tiles (RT even).
  int rt;
  if (a.epi == kEpiSwiglu) {
    rt = (mt == 1 && a.seg[0].n / 32 >= 2 * sms) ? 4 : 2;
  } else {
    rt = rows / 64 >= 2 * sms && mt == 1 ? 4 : (rows / 32 >= 2 * sms ? 2 : 1);
  }
  int n_ctas = 0;
  if (a.epi == kEpiSwiglu) {
    n_ctas = (a.seg[0].n + rt * 8 - 1) / (rt * 8);
  } else {
    for (int i = 0; i < a.n_seg; ++i) {
      a.seg_cta0[i] = n_ctas;
      n_ctas += (a.seg[i].n + rt * 16 - 1) / (rt * 16);
    }
    for (int i = a.n_seg; i < 4; ++i) a.seg_cta0[i] = n_ctas;
  }
  static void* err_word[64];
  if (dev >= 0 && dev < 64) {
    if (err_word[dev] == nullptr && device_error_address(&err_word[dev]) != cudaSuccess) {
      cudaGetLastError();
      err_word[dev] = nullptr;
    }
    a.err = static_cast<uint32_t*>(err_word[dev]);
  }
  switch (a.w_type) {
    case kWF16: return run_linear_t<kWF16>(a, rt, mt, n_ctas, s);
    case kWQ4_0: return run_linear_t<kWQ4_0>(a, rt, mt, n_ctas, s);
    case kWQ8_0: return run_linear_t<kWQ8_0>(a, rt, mt, n_ctas, s);
    case kWQ4_K: return run_linear_t<kWQ4_K>(a, rt, mt, n_ctas, s);
    case kWQ6_K: return run_linear_t<kWQ6_K>(a, rt, mt, n_ctas, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_swiglu(const __half* gate, const __half* up, __half* out, size_t n,
                          cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const size_t blocks = std::min<size_t>((n + 255) / 256, 148 * 16);
  swiglu_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(gate, up, out, n);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const __half* x, const __half* res, const __half* w, __half* h_out,
                           __half* out, int m, int k, float eps, cudaStream_t s) {
  if (m <= 0) return cudaSuccess;
  rmsnorm_kernel<<<static_cast<unsigned>(m), 256, 0, s>>>(x, res, w, h_out, out, k, eps);
  return cudaGetLastError();
}

}  // namespace kvc
