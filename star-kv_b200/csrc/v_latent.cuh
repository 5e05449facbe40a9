// v_latent.cuh — V path of the decode step: softmax weights x dequantised V
// latents, in latent space (the reorder branch of
// LlamaLoRaAttention_headwise.py:126-133 / model.py:482-487; bx_quant._bx_fwd,
// bx_quant.py:38-114), then the V up-projection once per head.
//
// The contraction runs on the tensor cores: int4 codes are dequantised
// (q*s + z, one fp16 rounding) straight into an MN-major fp16 A tile, the softmax
// weights of the block's heads form the K-major B tile, and D[channel, head]
// accumulates in TMEM over the split.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace starkv {

struct VParams {
  starkv_layout lay;
  const float* logits;   // (B, Hq, T) log2-domain logits (decode) ...
  const float* smax;     // (B, Hq, nsplit_k) maximum logit of each K split
  float* lsum;           // (B, Hq, nsplit) sum of exp2(logit - max) over each split (decode)
  const float* probs;    // ... or (B, Hq, T) probabilities (bx mode) when non-null
  const void* v_cache;
  const __half2* v_params;
  float* partial;        // decode: (B, Hq, nsplit, rv_max); bx mode: (B, Hq, R)
  int* err;
  int T, nsplit, nsplit_k, tps, rv_max;
  int ctiles;            // channel tiles of kVCtaRank per V block (grid.y = blocks * ctiles)
};

constexpr int kVThreads = 256;
constexpr int kVTile = 64;       // tokens per MMA step (K of the MMA)
constexpr int kVMaxHeads = 32;   // query heads of one V block (N of the MMA, padded to 32)
constexpr int kVCtaRank = 256;   // channels of a V block one CTA covers (two 128-row M tiles)
constexpr int kVMaxRank = 1024;  // V block rank (the reference's global V is one block)
constexpr int kVHeader = 1024;
constexpr float kVPScale = 4096.f;   // softmax weights enter the MMA as fp16(p * 2^12)

// A tile (one buffer): 2 M-tiles x [16 channel blocks of 8][8 token blocks of 8] fp16 core
// matrices (MN-major, no swizzle): element (c, l) of M-tile mt at
//   mt*16384 + (c%128/8)*1024 + (l/8)*128 + (l%8)*16 + (c%8)*2.
// B tile: [4 head blocks of 8][8 token blocks] (K-major): (g, l) at (g/8)*1024 + (l/8)*128 + (g%8)*16 + (l%8)*2.
constexpr int kVABytes = 2 * 16384;
constexpr int kVBBytes = 4096;

__host__ __device__ inline size_t v_smem_bytes() { return (size_t)kVHeader + 2 * (kVABytes + kVBBytes); }

// Instruction descriptor, kind::f16: A MN-major, B K-major, D f32, M=128, N=32.
__host__ __device__ constexpr uint32_t idesc_v() {
  return (1u << 4) | (1u << 15) | ((uint32_t)(32 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// 16 bytes of packed int4 codes (32 channels) -> 4 x 8 fp16 of q*s + z.
__device__ __forceinline__ void dequant32_i4(const uint4 w, __half2 s2, __half2 z2, uint4* out) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  const __half2 k1024 = __half2half2(__ushort_as_half((unsigned short)0x6400));
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint32_t x = ws[u] & 0x0F0F0F0Fu, y = (ws[u] >> 4) & 0x0F0F0F0Fu;
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // bytes: [x_i, -, y_i, -] -> fp16 pair (1024 + lo, 1024 + hi)
      uint32_t v = __byte_perm(x, y, (uint32_t)(i | ((4 + i) << 8)));
      v = (v & 0x000F000Fu) | 0x64006400u;
      __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), k1024);   // exact codes
      h = __hfma2(h, s2, z2);                                       // q*s + z, one rounding
      o[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    out[u] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// 32 unquantised latents -> 4 x 8 fp16.
template <typename LT>
__device__ __forceinline__ void convert32(const LT* src, uint4* out) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    __align__(16) __half h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(to_f32(src[u * 8 + e]));
    out[u] = *reinterpret_cast<uint4*>(h);
  }
}

// grid (nsplit, num_v_blocks * channel tiles of 256, B), 256 threads.  LT = latent type (unquantised) or uint8_t (int4 codes).
// D[c, g] = sum_l x_hat[l, c] * p[l, g] accumulates in TMEM (M = channels, N = heads) on the
// tensor cores over the split's tokens, 64 tokens per step, double-buffered.
template <typename LT, bool QUANT>
__global__ void __launch_bounds__(kVThreads) v_latent_kernel(const __grid_constant__ VParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const starkv_layout& lay = p.lay;
  const int split = blockIdx.x, b = blockIdx.z;
  const int blk = blockIdx.y / p.ctiles, ct = blockIdx.y % p.ctiles;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int qh0 = lay.v_first_kv[blk] * qpk;
  const int Gv = lay.v_num_kv[blk] * qpk;
  const int c_lo = ct * kVCtaRank;                                  // first channel of this CTA
  if (c_lo >= lay.v_rank[blk]) return;
  const int r = min(kVCtaRank, lay.v_rank[blk] - c_lo);            // channels of this CTA
  const int vcol = lay.v_col[blk] + c_lo;                           // global column of channel 0
  const int R = lay.v_rank_total;
  const int NQ = r >> 5;                 // 32-channel groups
  const int MT = (r + 127) >> 7;         // 128-channel M-tiles
  const int t_begin = split * p.tps, t_end = min(p.T, t_begin + p.tps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kVTile - 1) / kVTile : 0;

  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(smem);         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 64);
  volatile int* s_fail = reinterpret_cast<volatile int*>(smem + 68);
  float* s_mx = reinterpret_cast<float*>(smem + 256);             // [32]
  uint8_t* Abuf = smem + kVHeader;                                 // [2][kVABytes]
  uint8_t* Bbuf = Abuf + 2 * kVABytes;                             // [2][kVBBytes]

  // zero both A/B buffers once: padding channels / heads stay zero
  for (int e = tid; e < (2 * (kVABytes + kVBBytes)) / 16; e += kVThreads)
    reinterpret_cast<uint4*>(Abuf)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    mbar_init(mma_bar + 0, 1);
    mbar_init(mma_bar + 1, 1);
    *s_fail = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  for (int gw = warp; !p.probs && gw < Gv; gw += kVThreads / 32) {
    const int qh = qh0 + gw;
    float m = kNegBig;
    for (int s = lane; s < p.nsplit_k; s += 32) m = fmaxf(m, p.smax[((int64_t)b * Hq + qh) * p.nsplit_k + s]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_mx[gw] = m;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- per-thread work items of one 64-token tile
  // codes: item i -> token lo = i%8 + 8*(i/(8*NQ)), group q = (i/8)%NQ   (NQ*64 items)
  // weights: item i < 8*Gv -> head g = i/8, tokens 8*(i%8) .. +7
  const int n_items = NQ * kVTile;
  constexpr int kMaxItems = (kVCtaRank / 32) * kVTile / kVThreads;   // 2
  constexpr int CB = QUANT ? 16 : 32 * (int)sizeof(LT);              // bytes of 32 channels
  constexpr int CW = CB / 16;                                         // uint4 per item
  uint4 cw[kMaxItems][CW];
  __half2 sz[kMaxItems];
  float lg[8];
  float psum = 0.f;      // this thread's share of sum exp2(logit - max) (decode)

  auto load_tile = [&](int t) {
    const int t0 = t_begin + t * kVTile;
#pragma unroll
    for (int it = 0; it < kMaxItems; ++it) {
      const int i = tid + it * kVThreads;
      if (i < n_items) {
        const int lo = (i & 7) + 8 * (i / (8 * NQ)), q = (i >> 3) % NQ;
        const int l = t0 + lo;
        if (l < t_end) {
          const int64_t row = (int64_t)b * lay.capacity + l;
          if constexpr (QUANT) {
            cw[it][0] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.v_cache) + row * (R / 2) +
                                                        vcol / 2 + q * 16);
            sz[it] = p.v_params[row * (R / 32) + vcol / 32 + q];
          } else {
            const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const LT*>(p.v_cache) + row * R + vcol + q * 32);
#pragma unroll
            for (int u = 0; u < CW; ++u) cw[it][u] = src[u];
          }
        } else {
#pragma unroll
          for (int u = 0; u < CW; ++u) cw[it][u] = make_uint4(0u, 0u, 0u, 0u);
          sz[it] = __floats2half2_rn(0.f, 0.f);
        }
      }
    }
    if (tid < 8 * Gv) {
      const int g = tid >> 3, l0 = t0 + 8 * (tid & 7);
      const int64_t base = ((int64_t)b * Hq + qh0 + g) * p.T;
      const float* src = p.probs ? p.probs : p.logits;
#pragma unroll
      for (int e = 0; e < 8; ++e) lg[e] = (l0 + e < t_end) ? src[base + l0 + e] : 0.f;
    }
  };

  auto store_tile = [&](int t, int buf) {
    uint8_t* A = Abuf + buf * kVABytes;
    uint8_t* Bm = Bbuf + buf * kVBBytes;
#pragma unroll
    for (int it = 0; it < kMaxItems; ++it) {
      const int i = tid + it * kVThreads;
      if (i < n_items) {
        const int lo = (i & 7) + 8 * (i / (8 * NQ)), q = (i >> 3) % NQ;
        uint4 o[4];
        if constexpr (QUANT) {
          dequant32_i4(cw[it][0], __half2half2(__low2half(sz[it])), __half2half2(__high2half(sz[it])), o);
        } else {
          convert32<LT>(reinterpret_cast<const LT*>(&cw[it][0]), o);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = q * 32 + u * 8;
          *reinterpret_cast<uint4*>(A + (c >> 7) * 16384 + ((c & 127) >> 3) * 1024 + (lo >> 3) * 128 + (lo & 7) * 16) = o[u];
        }
      }
    }
    if (tid < 8 * Gv) {
      const int g = tid >> 3, kb = tid & 7;
      const int l0 = t_begin + t * kVTile + 8 * kb;
      __align__(16) __half h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float pv = 0.f;
        if (l0 + e < t_end) {
          if (p.probs) {
            pv = lg[e] * kVPScale;
          } else {
            const float x = exp2f(lg[e] - s_mx[g]);
            psum += x;
            pv = x * kVPScale;
          }
        }
        h[e] = __float2half_rn(pv);
      }
      *reinterpret_cast<uint4*>(Bm + (g >> 3) * 1024 + kb * 128 + (g & 7) * 16) = *reinterpret_cast<uint4*>(h);
    }
  };

  constexpr uint32_t IDESC = idesc_v();
  if (ntiles > 0) load_tile(0);
  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t >= 2) {
      // the MMAs of tile t-2 read this buffer
      int fail = !mbar_wait(mma_bar + buf, (uint32_t)(((t - 2) >> 1) & 1));
      if (fail) { record_error(p.err, kDevWaitMma); *s_fail = 1; }
    }
    if (__syncthreads_or(*s_fail)) break;
    store_tile(t, buf);
    if (t + 1 < ntiles) load_tile(t + 1);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(Abuf + buf * kVABytes), b0 = smem_u32(Bbuf + buf * kVBBytes);
      for (int mt = 0; mt < MT; ++mt)
        for (int ks = 0; ks < kVTile / 16; ++ks)
          mma_f16_ss(tmem + mt * 32, smem_desc(a0 + mt * 16384 + ks * 256, 128, 1024),
                     smem_desc(b0 + ks * 256, 128, 1024), IDESC, (t > 0 || ks > 0) ? 1u : 0u);
      mma_commit(mma_bar + buf);
    }
  }
  // ---- split sums of the exponentials (threads 8g .. 8g+7 hold head g; channel tile 0 writes)
  if (!p.probs && !*s_fail) {
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    if (ct == 0 && tid < 8 * Gv && (tid & 7) == 0)
      p.lsum[((int64_t)b * Hq + qh0 + (tid >> 3)) * p.nsplit + split] = psum;
  }
  // ---- wait for the last MMAs, read D[c, g] and write the partials
  if (tid == 0 && ntiles > 0 && !*s_fail) {
    const int t = ntiles - 1;
    if (!mbar_wait(mma_bar + (t & 1), (uint32_t)((t >> 1) & 1))) { record_error(p.err, kDevWaitMma); *s_fail = 1; }
  }
  __syncthreads();
  tc_fence_after();
  if (warp < 4 * MT && !*s_fail) {
    const int mt = warp >> 2, cq = warp & 3;
    const int c = mt * 128 + cq * 32 + lane;
    float d[32];
    if (ntiles > 0) {
      tmem_ld16x2(tmem + ((uint32_t)(cq * 32) << 16) + mt * 32, tmem + ((uint32_t)(cq * 32) << 16) + mt * 32 + 16, d,
                  d + 16);
    } else {
#pragma unroll
      for (int g = 0; g < 32; ++g) d[g] = 0.f;
    }
    if (c < r) {
#pragma unroll
      for (int g = 0; g < kVMaxHeads; ++g) {
        if (g < Gv) {
          const int qh = qh0 + g;
          const float v = d[g] * (1.f / kVPScale);
          if (p.probs)
            p.partial[((int64_t)b * Hq + qh) * R + vcol + c] = v;
          else
            p.partial[(((int64_t)b * Hq + qh) * p.nsplit + split) * p.rv_max + c_lo + c] = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// Merge the split partials and apply the V up-projection once per head:
//   out[b, h, d] = sum_c (sum_s partial[b, h, s, c]) * U_v[kv * 128 + d, vcol + c]
// grid (Hq, B), 128 threads.
struct CombineParams {
  starkv_layout lay;
  const float* partial;
  const float* lsum;     // (B, Hq, nsplit) split sums of the softmax exponentials
  const void* v_u;
  void* out;
  int w_dtype, out_dtype, nsplit, rv_max;
};

__global__ void __launch_bounds__(128) combine_kernel(const __grid_constant__ CombineParams p) {
  __shared__ float o_lat[kVMaxRank];
  const starkv_layout& lay = p.lay;
  const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads, kv = qh / qpk;
  int blk = 0;
  while (blk + 1 < lay.num_v_blocks && lay.v_first_kv[blk + 1] <= kv) ++blk;
  const int r = lay.v_rank[blk], vcol = lay.v_col[blk], R = lay.v_rank_total;
  __shared__ float s_inv;
  if (tid < 32) {
    float L = 0.f;
    for (int k = tid; k < p.nsplit; k += 32) L += p.lsum[((int64_t)b * Hq + qh) * p.nsplit + k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (tid == 0) s_inv = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const float inv = s_inv;
  // split sums: warp w adds splits w, w + 4, ... for channels lane + 32i (coalesced
  // rows, up to eight independent loads in flight per lane), then the four warps'
  // sums meet in shared memory in a fixed order (the result does not depend on timing)
  __shared__ float part[4][kVMaxRank];
  {
    const int w = tid >> 5, ln = tid & 31;
    const float* base = p.partial + ((int64_t)b * Hq + qh) * p.nsplit * p.rv_max;
    for (int c0 = 0; c0 < r; c0 += 256) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int k = w; k < p.nsplit; k += 4) {
        const float* src = base + (int64_t)k * p.rv_max + c0 + ln;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (c0 + ln + 32 * i < r) acc[i] += src[32 * i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c0 + ln + 32 * i < r) part[w][c0 + ln + 32 * i] = acc[i];
    }
  }
  __syncthreads();
  for (int c = tid; c < r; c += 128) o_lat[c] = (((part[0][c] + part[1][c]) + part[2][c]) + part[3][c]) * inv;
  __syncthreads();
  // out[d] = sum_c o_lat[c] * U_v[kv * 128 + d, vcol + c]: warp w takes the rows
  // d = w, w + 4, ...; lane l the 8 consecutive channels 8l + 256k of the row (one
  // 16-byte load for 16-bit weights; its 8 latent values stay in registers), then
  // a shuffle reduction.
  const int warp = tid >> 5, lane = tid & 31;
  const bool vec = p.w_dtype != STARKV_F32 && (R % 8) == 0 && (vcol % 8) == 0 && (r % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(p.v_u) & 15) == 0;
  float ol[kVMaxRank / 256][8];
#pragma unroll
  for (int k = 0; k < kVMaxRank / 256; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = lane * 8 + 256 * k + e;
      ol[k][e] = c < r ? o_lat[c] : 0.f;
    }
  // four rows per iteration (d, d + 4, d + 8, d + 12): their loads in flight together
  for (int d0 = warp; d0 < 128; d0 += 16) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kVMaxRank / 256; ++k) {
      const int c = lane * 8 + 256 * k;
      if (c >= r) break;
      if (vec) {
        uint4 w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          w[q] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.v_u) +
                                                 ((int64_t)kv * 128 + d0 + 4 * q) * R + vcol + c);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t ws[4] = {w[q].x, w[q].y, w[q].z, w[q].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float lo, hi;
            if (p.w_dtype == STARKV_F16) {
              const __half2 h = *reinterpret_cast<const __half2*>(&ws[e]);
              lo = __low2float(h);
              hi = __high2float(h);
            } else {
              lo = __uint_as_float(ws[e] << 16);
              hi = __uint_as_float(ws[e] & 0xFFFF0000u);
            }
            acc[q] = fmaf(ol[k][2 * e], lo, acc[q]);
            acc[q] = fmaf(ol[k][2 * e + 1], hi, acc[q]);
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int64_t urow = ((int64_t)kv * 128 + d0 + 4 * q) * R + vcol;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c + e < r) acc[q] = fmaf(ol[k][e], load_as_f32(p.v_u, p.w_dtype, urow + c + e), acc[q]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float a = acc[q];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) store_from_f32(p.out, p.out_dtype, ((int64_t)b * Hq + qh) * 128 + d0 + 4 * q, a);
    }
  }
}

// ============================================================================
// Decode V path, streaming form (int4 latents): CTA = (V split, sequence b), all
// V blocks and all query heads of the layer, one CTA per SM, 512 threads.
//
// A 64-token tile of one sequence is one contiguous block of int4 codes
// (64 x R/2 bytes) and one of fp16 (scale, zero) pairs (64 x R/8 bytes) in HBM:
//   producer warp:  1-D bulk copies of both into a ring of shared-memory stages,
//                   and an L2 prefetch of the tile's logits;
//   dequant warps (12, six pairs): per "M unit" = 128 consecutive channels of the
//                   whole latent row, q*s + z (one fp16 rounding, channels in the
//                   order [0,4,1,5,2,6,3,7] within every 8) into one of 6 MN-major
//                   A tiles (128 channels x 64 tokens); lane 0 of a pair's first
//                   warp issues the unit's 4 tcgen05.mma (M=128, N=NP >= Hq,
//                   K=16) into the unit's accumulator D[channel, head] in TMEM.
//                   With U >= 6 units pair p takes the units p, p + 6, ... of every
//                   tile; with U < 6 (a head shard) each unit gets floor(6 / U)
//                   pairs, replica j taking the tiles t = j mod replicas into its
//                   own accumulator, summed in the epilogue;
//   prob warps (2): p = exp2(logit - M_h) for every head (M_h = maximum over the
//                   K splits), fp16(p * 2^12) into a K-major B tile of all heads
//                   (two per replica, tile t in buffer t mod 2 * replicas), and the
//                   running sum of p.
// At the end the dequant warps read the accumulators and write the split
// partials of each channel's own V block heads; the prob warps write the split
// sums of p.  The combine kernel divides by the total sum.
// ============================================================================
constexpr int kV2Threads = 512;
constexpr int kV2Tile = 64;
constexpr int kV2Abufs = 6;        // one per dequant warp pair
constexpr int kV2ABytes = 16384;     // 128 channels x 64 tokens fp16
constexpr int kV2Header = 2048;
constexpr int kV2MaxStages = 4;
constexpr int kV2MaxUnits = 64;
constexpr int kV2MaxHeads = 64;

struct V2Params {
  starkv_layout lay;
  const float* logits;   // (B, Hq, T) log2-domain logits
  const float* smax;     // (B, Hq, nsplit_k) maximum logit of each K split
  float* lsum;           // (B, Hq, nsplit) sum of exp2(logit - max) over each V split
  const uint8_t* v_cache;
  const uint8_t* v_params;
  float* partial;        // (B, Hq, nsplit, rv_max)
  int* err;
  int T, nsplit, nsplit_k, tps, rv_max;
  int nstages, stage_bytes, b_bytes;
#ifdef STARKV_KTRACE
  long long* trace;      // diagnostic builds only: clock64 per (tile of CTA (0, 0), field)
#endif
};
#ifdef STARKV_KTRACE
#define VTRACE(t, f)                                                                                   \
  do {                                                                                                 \
    if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && (t) < 256) p.trace[(t) * 8 + (f)] = clock64(); \
  } while (0)
#else
#define VTRACE(t, f) do { } while (0)
#endif


// Dequant warp pairs per tile and accumulator replicas: with U = ceil(R / 128) M
// units, U >= 6 keeps all six pairs on every tile (pair p takes units p, p + 6, ...);
// U < 6 gives each unit floor(6 / U) pairs, replica j taking the tiles t with
// t % replicas == j into its own accumulator (summed at the end), so a layer
// with few V channels (a head shard) still dequantises with most warps.
__host__ __device__ inline int v2_tile_pairs(int R) { const int u = (R + 127) / 128; return u < 6 ? u : 6; }
__host__ __device__ inline int v2_replicas(int R) { const int u = (R + 127) / 128; return u < 6 ? 6 / u : 1; }
// B tiles (probabilities): two per replica, tile t in buffer t % (2 * replicas), so
// the previous use of a pair's buffer was that same pair's tile (no pair can run
// a barrier phase ahead of the prob warps).
__host__ __device__ inline int v2_bbufs(int R) { return 2 * v2_replicas(R); }

__host__ __device__ inline int v2_stage_bytes(int R) {
  return ((kV2Tile * (R / 2) + kV2Tile * (R / 8) + 32) + 127) & ~127;
}

// End (exclusive) of the staged parameter bytes of a tile whose rows end at byte
// `end`: rounded up to 16 bytes unless that would pass the buffer's end.
__host__ __device__ inline int64_t v2_param_end(int64_t end, int64_t total) {
  const int64_t up = (end + 15) & ~(int64_t)15;
  return up <= total ? up : (end & ~(int64_t)15);
}
__host__ __device__ inline size_t v2_smem_bytes(int nstages, int stage_bytes, int b_bytes, int nbb) {
  return (size_t)kV2Header + (size_t)nstages * stage_bytes + (size_t)kV2Abufs * kV2ABytes + (size_t)nbb * b_bytes;
}

// 32 int4 codes (16 bytes, even channel in the low nibble) -> 4 x 8 fp16 of q*s + z
// in the channel order [0, 4, 1, 5, 2, 6, 3, 7] within every 8 (one LOP3 puts two
// nibbles under the 0x6400 exponent; the subtraction of 1024 (or of 1024 for a
// nibble scaled by 16) is exact, the fused q*s + z one rounding; s16 = s / 16).
__device__ __forceinline__ void dequant32_i4_perm(const uint4 w, __half2 s2, __half2 s16, __half2 z2, uint4* out) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  const __half2 k1024 = __half2half2(__ushort_as_half((unsigned short)0x6400));
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint32_t w8 = ws[u] >> 8;
    uint32_t a = (ws[u] & 0x000F000Fu) | 0x64006400u;   // channels 0, 4
    uint32_t c = (ws[u] & 0x00F000F0u) | 0x64006400u;   // channels 1, 5 (x16)
    uint32_t e = (w8 & 0x000F000Fu) | 0x64006400u;      // channels 2, 6
    uint32_t g = (w8 & 0x00F000F0u) | 0x64006400u;      // channels 3, 7 (x16)
    __half2 ha = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&a), k1024), s2, z2);
    __half2 hc = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&c), k1024), s16, z2);
    __half2 he = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&e), k1024), s2, z2);
    __half2 hg = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&g), k1024), s16, z2);
    out[u] = make_uint4(*reinterpret_cast<uint32_t*>(&ha), *reinterpret_cast<uint32_t*>(&hc),
                        *reinterpret_cast<uint32_t*>(&he), *reinterpret_cast<uint32_t*>(&hg));
  }
}

// Channel held at position j (0..7) of a dequant32_i4_perm 8-channel row.
__host__ __device__ constexpr int v_perm8(int j) { return (j >> 1) + 4 * (j & 1); }

// Dequantise one M unit (GC groups of 32 channels x 64 tokens) into an MN-major A tile.
// Item it = (token, group); 8 consecutive lanes = 8 tokens of one group, so every
// 16-byte store phase covers 128 contiguous bytes.  pl = lane within the warp pair.
template <int GC>
__device__ __forceinline__ void v2_dequant_unit(const uint8_t* codes, const uint8_t* pars, const uint8_t* gpars,
                                                int pdelta, int pcopied, int c0, int nrows, int code_row,
                                                int par_row, uint8_t* A, int pl) {
#pragma unroll
  for (int k = 0; k < GC; ++k) {
    const int row8 = (pl >> 3) + 8 * k;
    const int grp = row8 % GC, l = (row8 / GC) * 8 + (pl & 7);
    uint4 o[4] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u),
                  make_uint4(0u, 0u, 0u, 0u)};
    if (l < nrows) {
      const uint4 w = *reinterpret_cast<const uint4*>(codes + l * code_row + (c0 >> 1) + grp * 16);
      const int po = l * par_row + ((c0 >> 5) + grp) * 4;
      const uint32_t pz = pdelta + po + 4 <= pcopied ? *reinterpret_cast<const uint32_t*>(pars + pdelta + po)
                                                     : *reinterpret_cast<const uint32_t*>(gpars + po);
      const __half2 sz = *reinterpret_cast<const __half2*>(&pz);
      const __half2 s2 = __half2half2(__low2half(sz));
      dequant32_i4_perm(w, s2, __hmul2(s2, __half2half2(__float2half_rn(0.0625f))), __half2half2(__high2half(sz)), o);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      *reinterpret_cast<uint4*>(A + (grp * 4 + u) * 1024 + (l >> 3) * 128 + (l & 7) * 16) = o[u];
  }
}

// 8 int4 codes (4 bytes, even channel in the low nibble) -> 8 fp16 of q*s + z.
__device__ __forceinline__ uint4 dequant8_i4(uint32_t w, __half2 s2, __half2 z2) {
  const __half2 k1024 = __half2half2(__ushort_as_half((unsigned short)0x6400));
  const uint32_t x = w & 0x0F0F0F0Fu, y = (w >> 4) & 0x0F0F0F0Fu;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t v = __byte_perm(x, y, (uint32_t)(i | ((4 + i) << 8)));
    v = (v & 0x000F000Fu) | 0x64006400u;
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), k1024);
    h = __hfma2(h, s2, z2);
    o[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int NP>
__global__ void __launch_bounds__(kV2Threads, 1) v_decode_kernel(const __grid_constant__ V2Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const starkv_layout& lay = p.lay;
  const int split = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int R = lay.v_rank_total;
  const int t_begin = split * p.tps, t_end = min(p.T, t_begin + p.tps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kV2Tile - 1) / kV2Tile : 0;
  const int NS = p.nstages;
  const int NB = v2_bbufs(lay.v_rank_total);      // B tiles
  const int code_row = R / 2, par_row = R / 8;
  const int64_t ptotal = (int64_t)lay.batch * lay.capacity * par_row;   // bytes of the parameter buffer

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 1536);
  uint64_t* st_full = bars;            // [4]
  uint64_t* st_empty = bars + 4;       // [4]  the active dequant warps
  uint64_t* a_full = bars + 8;         // [6]  the slot's dequant warp pair
  uint64_t* a_empty = bars + 14;       // [6]  commit of the pair's MMAs
  uint64_t* b_full = bars + 20;        // [NB <= 12]  2 prob warps
  uint64_t* b_empty = bars + 32;       // [NB]  commits of the tile's pairs
  uint64_t* fin_bar = bars + 44;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 192);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 196);
  int* s_nunits = reinterpret_cast<int*>(smem + 200);
  uint8_t* s_cblk = smem + 256;                               // [kV2MaxUnits * 4] V block of each 32-channel group
  float* s_mx = reinterpret_cast<float*>(smem + 512);         // [64] softmax maximum per head
  float* s_ps = reinterpret_cast<float*>(smem + 768);         // [2][64] prob-warp sums
  uint8_t* Ssm = smem + kV2Header;
  uint8_t* Asm = Ssm + (size_t)NS * p.stage_bytes;
  uint8_t* Bsm = Asm + (size_t)kV2Abufs * kV2ABytes;

  if (tid == 0) {
    for (int k = 0; k < kV2MaxStages; ++k) {
      mbar_init(st_full + k, 1);
      mbar_init(st_empty + k, 2 * v2_tile_pairs(R) * v2_replicas(R));
    }
    for (int k = 0; k < kV2Abufs; ++k) {
      mbar_init(a_full + k, 2);        // the slot's warp pair
      mbar_init(a_empty + k, 1);
    }
    for (int k = 0; k < v2_bbufs(R); ++k) {
      mbar_init(b_full + k, 2);
      mbar_init(b_empty + k, v2_tile_pairs(R));
    }
    mbar_init(fin_bar, v2_tile_pairs(R) * v2_replicas(R));
    *s_abort = 0;
    for (int j = 0; j < lay.num_v_blocks; ++j)
      for (int c = lay.v_col[j]; c < lay.v_col[j] + lay.v_rank[j]; c += 32) s_cblk[c >> 5] = (uint8_t)j;
    *s_nunits = (R + 127) / 128;
    fence_mbar_init();
  }
  // zero the B tiles once: padded heads stay zero
  for (int e = tid; e < (v2_bbufs(R) * p.b_bytes) / 16; e += kV2Threads) reinterpret_cast<uint4*>(Bsm)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (warp == 0) {                     // one CTA per SM: all 512 columns
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int MU = *s_nunits;
  auto fail = [&](int code) {
    record_error(p.err, code);
    *s_abort = 1;
  };

  if (warp == 0) {
    // ============================================================ producer
    if (lane == 0) {
      int issued = 0;
      for (int t = 0; t < ntiles; ++t, issued = t) {
        if (*s_abort) break;
        const int s = t % NS;
        if (!mbar_wait(st_empty + s, (uint32_t)(((t / NS) & 1) ^ 1))) { fail(kDevWaitCopy); break; }
        const int t0 = t_begin + t * kV2Tile;
        const int nrows = min(kV2Tile, t_end - t0);
        const int64_t row0 = (int64_t)b * lay.capacity + t0;
        const uint32_t cb = (uint32_t)(nrows * code_row);
        // parameters: [row0, row0 + nrows) rows widened to 16-byte boundaries, the end
        // rounded down only at the end of the buffer (that tail is read from global
        // by the dequant warps)
        const int64_t pstart = row0 * par_row, pa = pstart & ~(int64_t)15;
        const int64_t pend = v2_param_end(pstart + (int64_t)nrows * par_row, ptotal);
        const uint32_t pb = pend > pa ? (uint32_t)(pend - pa) : 0u;
        mbar_arrive_expect_tx(st_full + s, cb + pb);
        uint8_t* dst = Ssm + (size_t)s * p.stage_bytes;
        bulk_g2s(dst, p.v_cache + row0 * code_row, cb, st_full + s);
        VTRACE(t, 0);
        if (pb) bulk_g2s(dst + kV2Tile * code_row, p.v_params + pa, pb, st_full + s);
        // the tile's logits (one row of nrows floats per head) into L2 for the prob
        // warps: the 16-byte-aligned span inside each row (a hint; the ends are
        // loaded from HBM)
        for (int h = 0; h < Hq; ++h) {
          const uintptr_t a0 = reinterpret_cast<uintptr_t>(p.logits + ((int64_t)b * Hq + h) * p.T + t0);
          const uintptr_t lo = (a0 + 15) & ~(uintptr_t)15, hi = (a0 + (uintptr_t)nrows * 4) & ~(uintptr_t)15;
          if (hi > lo) bulk_prefetch_l2(reinterpret_cast<const void*>(lo), (uint32_t)(hi - lo));
        }
      }
      for (int t = max(0, issued - NS); t < issued; ++t)
        if (!mbar_wait(st_full + (t % NS), (uint32_t)((t / NS) & 1))) { fail(kDevWaitCopy); break; }
    }
    __syncwarp();
  } else if (warp == 1) {
    // (warp 1 has no role: the dequant warp pairs issue their own units' MMAs)
  } else if (warp < 4) {
    // ============================================================ prob warps
    const int pw = warp - 2, pt = tid - 64;
    for (int h = pt; h < Hq; h += 64) {
      float m = kNegBig;
      for (int s = 0; s < p.nsplit_k; ++s) m = fmaxf(m, p.smax[((int64_t)b * Hq + h) * p.nsplit_k + s]);
      s_mx[h] = m;
    }
    named_bar_sync(1, 64);
    const int G8 = (Hq + 7) >> 3;                  // groups of 8 heads (the last may be partial)
    constexpr int QG = NP / 8;                     // head groups a B tile holds
    // destination of this lane's (head, 8-token block) in a B tile, per head group
    int dstoff[QG];
    float mh[QG], psum[QG];
#pragma unroll
    for (int q = 0; q < QG; ++q) {
      dstoff[q] = 0;
      mh[q] = 0.f;
      psum[q] = 0.f;
      if (q < G8) {
        const int g = q * 8 + (lane & 7);
        dstoff[q] = (g >> 3) * 1024 + (g & 7) * 16;
        mh[q] = g < Hq ? s_mx[g] : 0.f;
      }
    }
    const int kb = (lane >> 3) + 4 * pw;           // 8-token block of the tile
    auto load_lg = [&](int t, float (&lg)[QG][8]) {
      const int l0 = t_begin + t * kV2Tile + kb * 8;
#pragma unroll
      for (int q = 0; q < QG; ++q)
        if (q < G8) {
          const float* src = p.logits + ((int64_t)b * Hq + q * 8 + (lane & 7)) * p.T + l0;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            lg[q][e] = (q * 8 + (lane & 7) < Hq && t < ntiles && l0 + e < t_end) ? __ldg(src + e) : kNegBig;
        }
    };
    // the next tile's logits are loaded while this tile's weights are formed
    float lg[QG][8], lgn[QG][8];
    load_lg(0, lg);
    bool ok = true;
    int tb = 0;                                    // B tile t % NB
    uint32_t bph = 0;                              // parity of its (t / NB)-th use
    for (int t = 0; t < ntiles; ++t) {
      if (t > 0 && ++tb == NB) { tb = 0; bph ^= 1; }
      if (*s_abort) break;
      const int l0 = t_begin + t * kV2Tile + kb * 8;
      load_lg(t + 1, lgn);
      if (!mbar_wait(b_empty + tb, bph ^ 1)) { ok = false; break; }
      uint8_t* Bt = Bsm + tb * p.b_bytes + kb * 128;
#pragma unroll
      for (int q = 0; q < QG; ++q)
        if (q < G8) {
          __align__(16) __half hv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float x = (q * 8 + (lane & 7) < Hq && l0 + e < t_end) ? exp2f(lg[q][e] - mh[q]) : 0.f;
            psum[q] += x;
            hv[e] = __float2half_rn(x * kVPScale);
          }
          *reinterpret_cast<uint4*>(Bt + dstoff[q]) = *reinterpret_cast<uint4*>(hv);
        }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_full + tb);
      if (tid == 64) VTRACE(t, 2);
#pragma unroll
      for (int q = 0; q < QG; ++q)
#pragma unroll
        for (int e = 0; e < 8; ++e) lg[q][e] = lgn[q][e];
    }
    if (!ok) fail(kDevWaitMma);
    // sum over the 4 lanes of a head (same lane & 7), then over the two warps
#pragma unroll
    for (int q = 0; q < QG; ++q) {
      float v = psum[q];
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (q < G8 && lane < 8) s_ps[pw * 64 + q * 8 + lane] = v;
    }
    named_bar_sync(1, 64);
    if (!*s_abort)
      for (int h = pt; h < Hq; h += 64) p.lsum[((int64_t)b * Hq + h) * p.nsplit + split] = s_ps[h] + s_ps[64 + h];
  } else {
    // ============================================================ dequant warps
    // Warp pair p (p < TP * RF active pairs, TP = pairs per tile, RF = replicas)
    // takes the units m = p % TP, m + 6, ... of the tiles t with t % RF == p / TP,
    // into A slots p, p + TP * RF, ... (a pair keeps several tiles in flight when
    // fewer than six pairs work).  Per tile it dequantises each of its units into
    // a slot and lane 0 of its first warp issues that unit's MMAs into the
    // replica's accumulator (one thread waits about as long per tcgen05.mma as
    // the tensor core takes for one, so several issuing pairs keep it busy); an
    // accumulator therefore always grows in tile order.
    const int dw = warp - 4;                       // 0..11
    const int pair = dw >> 1, pl = (dw & 1) * 32 + lane;
    const bool issuer = (dw & 1) == 0 && lane == 0;
    const int TP = v2_tile_pairs(R), RF = v2_replicas(R), NACT = TP * RF;
    const int SPP = kV2Abufs / NACT;               // A slots of each active pair
    const int rep_j = pair / TP, m0 = pair % TP;
    // Rotating tail: with U = 6q + rem units (q >= 1, 0 < rem < 6), units below 6q keep
    // their owner pairs and tail unit i goes to pair (t * rem + i) mod 6 in tile t, into
    // that pair's own accumulator for it (summed in the epilogue), so every pair
    // dequantises about U / 6 units per tile (when the 6q + 6 rem accumulators fit TMEM).
    const int q6 = (MU / 6) * 6, rem = MU - q6;
    const bool TAIL = RF == 1 && q6 > 0 && rem > 0 && (q6 + 6 * rem) * NP <= 512;
    constexpr uint32_t IDESC = (1u << 4) | (1u << 15) | ((uint32_t)(NP >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    int ks = 0;                                    // slot index of the next unit (slot pair + NACT * ks)
    uint32_t kph = 0;                              // its use parity
    bool ok = true;
    const bool active = pair < NACT;
    // every active warp passes every stage (so none falls a barrier phase behind)
    // and works on its replica's tiles
    int s = 0, sph = 0, tr = 0;                    // stage and its parity, t % RF
    int tb = 0;                                    // B tile t % NB and the parity of its use
    uint32_t bph = 0;
    int trot = 0;                                  // (t * rem) mod 6
    uint32_t tinit = 0;                            // tail accumulators of this pair already written
    for (int t = 0; active && t < ntiles && ok; ++t, tr = (tr + 1 == RF) ? 0 : tr + 1) {
      if (t > 0) {
        if (++s == NS) { s = 0; sph ^= 1; }
        if (++tb == NB) { tb = 0; bph ^= 1; }
        trot = (trot + rem) % 6;
      }
      if (*s_abort) break;
      if (!mbar_wait(st_full + s, (uint32_t)sph)) { ok = false; break; }
      if (tr != rep_j) {
        __syncwarp();
        if (lane == 0) mbar_arrive(st_empty + s);
        continue;
      }
      if (dw == 0 && lane == 0) VTRACE(t, 1);
      const uint8_t* codes = Ssm + (size_t)s * p.stage_bytes;
      const uint8_t* pars = codes + kV2Tile * code_row;
      const int t0 = t_begin + t * kV2Tile;
      const int nrows = min(kV2Tile, t_end - t0);
      const int64_t pstart = ((int64_t)b * lay.capacity + t0) * par_row;
      const int pdelta = (int)(pstart & 15);                // stage byte of parameter row 0
      const int64_t pend = v2_param_end(pstart + (int64_t)nrows * par_row, ptotal);
      const int pcopied = pend > (pstart & ~(int64_t)15) ? (int)(pend - (pstart & ~(int64_t)15)) : 0;
      const uint8_t* gpars = p.v_params + pstart;
      bool have_b = false;
      int own_m = m0, ti = 0;
      const int nown = TAIL ? q6 : MU;
      while (ok) {
        int m, dcol;                                         // unit, its accumulator's first column
        bool first;                                          // first tile into that accumulator
        if (own_m < nown) {
          m = own_m;
          own_m += kV2Abufs;
          dcol = (rep_j * TP + m) * NP;
          first = t == rep_j;
        } else {
          if (!TAIL) break;
          while (ti < rem && (trot + ti) % 6 != pair) ++ti;
          if (ti >= rem) break;
          m = q6 + ti;
          dcol = (q6 + pair * rem + ti) * NP;
          first = ((tinit >> ti) & 1u) == 0;
          tinit |= 1u << ti;
          ++ti;
        }
        const int k = pair + NACT * ks;                      // slot of this unit
        const uint32_t ph = kph;
        if (++ks == SPP) { ks = 0; kph ^= 1; }
        if (!mbar_wait(a_empty + k, ph ^ 1)) { ok = false; break; }
        const int c0 = m * 128;                              // first global channel of the M unit
        const int nch = min(128, R - c0);
        const int gc = nch >> 5;                             // 32-channel groups in the M tile
        uint8_t* A = Asm + k * kV2ABytes;
        switch (gc) {
          case 1: v2_dequant_unit<1>(codes, pars, gpars, pdelta, pcopied, c0, nrows, code_row, par_row, A, pl); break;
          case 2: v2_dequant_unit<2>(codes, pars, gpars, pdelta, pcopied, c0, nrows, code_row, par_row, A, pl); break;
          case 3: v2_dequant_unit<3>(codes, pars, gpars, pdelta, pcopied, c0, nrows, code_row, par_row, A, pl); break;
          default: v2_dequant_unit<4>(codes, pars, gpars, pdelta, pcopied, c0, nrows, code_row, par_row, A, pl); break;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + k);
        if (issuer) {
          bool good = mbar_wait(a_full + k, ph);            // both warps of the pair wrote the slot
          if (good && !have_b) good = mbar_wait(b_full + tb, bph);
          if (!good) {
            fail(kDevWaitMma);
          } else {
            have_b = true;
            tc_fence_after();
            const uint64_t ad = smem_desc(smem_u32(A), 128, 1024);
            const uint64_t bd = smem_desc(smem_u32(Bsm + tb * p.b_bytes), 128, 1024);
            const uint32_t d = tmem + (uint32_t)dcol;
#pragma unroll
            for (int kk = 0; kk < kV2Tile / 16; ++kk)
              mma_f16_ss(d, ad + (uint64_t)(kk * 16), bd + (uint64_t)(kk * 16), IDESC, (!first || kk > 0) ? 1u : 0u);
            mma_commit(a_empty + k);
          }
        }
        __syncwarp();
      }
      if (issuer) mma_commit(b_empty + tb);                 // this pair's reads of the tile's B are queued
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(st_empty + s);
      if (dw == 0 && lane == 0) VTRACE(t, 5);
    }
    if (issuer && active) mma_commit(fin_bar);              // arrives once this pair's MMAs retired
    if (!ok) fail(kDevWaitMma);
    // ---- epilogue: accumulators -> split partials (warp quarter = TMEM lanes)
    const bool have = ntiles > 0 && !*s_abort;
    if (have && !mbar_wait(fin_bar, 0)) fail(kDevWaitMma);
    tc_fence_after();
    const int q4 = warp & 3;
    for (int m = dw >> 2; m < MU; m += 3) {
      const int cg = m * 128 + q4 * 32 + (lane & ~7) + v_perm8(lane & 7);   // global channel of this lane's row
      const int blk = cg < R ? s_cblk[cg >> 5] : 0;
      const int Gv = lay.v_num_kv[blk] * qpk, qh0 = lay.v_first_kv[blk] * qpk;
      const int c = cg - lay.v_col[blk];                     // channel within the V block
      const bool rd = have && !*s_abort;
#pragma unroll
      for (int h = 0; h < NP; h += 16) {                     // 16 heads at a time
        float d[16];
#pragma unroll
        for (int g = 0; g < 16; ++g) d[g] = 0.f;
        // the unit's accumulators that received a tile: replica j of an owned unit
        // gets tiles j, j + RF, ...; pair cand's copy of tail unit i the tiles with
        // (t * rem + i) mod 6 == cand (a pattern of period <= 6)
        const bool tail_m = TAIL && m >= q6;
        const int ncand = tail_m ? 6 : RF;
        for (int cand = 0; rd && cand < ncand; ++cand) {
          bool use = false;
          int col;
          if (tail_m) {
            for (int tt = 0; tt < ntiles && tt < 6; ++tt) use |= (tt * rem + (m - q6)) % 6 == cand;
            col = (q6 + cand * rem + (m - q6)) * NP;
          } else {
            use = cand < ntiles;
            col = (cand * TP + m) * NP;
          }
          if (!use) continue;
          float e[16];
          tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(col + h), e);
#pragma unroll
          for (int g = 0; g < 16; ++g) d[g] += e[g];
        }
        if (cg < R) {
#pragma unroll
          for (int g = 0; g < 16; ++g)
            if (h + g >= qh0 && h + g < qh0 + Gv)
              p.partial[(((int64_t)b * Hq + h + g) * p.nsplit + split) * p.rv_max + c] = d[g] * (1.f / kVPScale);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace starkv
