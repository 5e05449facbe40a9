// quant.cuh — latent quantise / append kernels (replace the reference's missing
// quant_utils.quantize_r_split_int8_int4_packed and Cache.update's torch.cat).
//
// Quantiser specification (bit-exact, IEEE fp32, round-to-nearest-even):
//   K int8 symmetric per (sequence, KV head, channel):
//     s = fp16(absmax / 127), s = 1 where that is 0;  q = clamp(rint(x / s), -127, 127)
//   V int4 asymmetric per token, groups of 32 channels:
//     s = fp16((max - min) / 15), s = 1 where that is 0;  z = fp16(min);
//     q = clamp(rint((x - z) / s), 0, 15); two codes a byte, even channel low nibble
//     (the nibble order bx_quant.py:75-85 reads).
// No fast-math: __fdiv_rn / __fsub_rn / rintf keep the arithmetic exact.
#pragma once
#include "common.cuh"

namespace starkv {

// ---- K: per-channel scales over the prefill + codes for the prefill tokens.
// grid (Hkv, B, Z), block 256.  k_lat: (B, T, k_rank_total) latent dtype.  Every
// CTA of a (KV head, sequence) forms the same per-channel absmax over all T
// tokens (the re-reads come from L2), CTA z == 0 writes the scales, and CTA z
// quantises tokens [z*ceil(T/Z), (z+1)*ceil(T/Z)): the prompt's tokens spread
// over many SMs instead of one CTA per head.
template <typename LT>
__global__ void __launch_bounds__(256) k_prefill_quant_kernel(const starkv_layout lay, const LT* __restrict__ k_lat,
                                                              int T, int8_t* __restrict__ k_cache,
                                                              __half* __restrict__ k_scales) {
  const int kv = blockIdx.x, b = blockIdx.y;
  const int r = lay.k_rank[kv];
  const int K = lay.k_rank_total;
  const int col = threadIdx.x & 31, slot = threadIdx.x >> 5;
  __shared__ float red[8][STARKV_MAX_K_RANK];
  __shared__ float sc[STARKV_MAX_K_RANK];
  const LT* src = k_lat + (int64_t)b * T * K + lay.k_col[kv];
  for (int c0 = 0; c0 < r; c0 += 32) {
    const int c = c0 + col;
    float amax = 0.f;
    if (c < r)
      for (int t = slot; t < T; t += 8) amax = fmaxf(amax, fabsf(to_f32(src[(int64_t)t * K + c])));
    if (c < r) red[slot][c] = amax;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < r; c += blockDim.x) {
    float amax = red[0][c];
#pragma unroll
    for (int s = 1; s < 8; ++s) amax = fmaxf(amax, red[s][c]);
    __half h = __float2half_rn(__fdiv_rn(amax, 127.0f));
    if (__half2float(h) == 0.0f) h = __float2half_rn(1.0f);
    if (blockIdx.z == 0) k_scales[(int64_t)b * K + lay.k_col[kv] + c] = h;
    sc[c] = __half2float(h);
  }
  __syncthreads();
  const int chunk = (T + gridDim.z - 1) / gridDim.z;
  const int t0 = blockIdx.z * chunk, t1 = min(T, t0 + chunk);
  for (int t = t0 + slot; t < t1; t += 8)
    for (int c = col; c < r; c += 32) {
      float q = rintf(__fdiv_rn(to_f32(src[(int64_t)t * K + c]), sc[c]));
      q = fminf(fmaxf(q, -127.f), 127.f);
      k_cache[k_elem(lay, kv, b, t, c, 1)] = (int8_t)(int)q;
    }
}

// ---- K append with existing scales.  One thread per (b, t, channel of sum r).
template <typename LT>
__global__ void __launch_bounds__(256) k_append_quant_kernel(const starkv_layout lay, const LT* __restrict__ k_lat,
                                                             int T, int start, int8_t* __restrict__ k_cache,
                                                             const __half* __restrict__ k_scales) {
  const int K = lay.k_rank_total;
  const int64_t n = (int64_t)lay.batch * T * K;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int ch = (int)(e % K);
    const int64_t bt = e / K;
    const int t = (int)(bt % T), b = (int)(bt / T);
    int kv = 0;
    while (kv + 1 < lay.num_kv_heads && lay.k_col[kv + 1] <= ch) ++kv;
    const int c = ch - lay.k_col[kv];
    const float s = __half2float(k_scales[(int64_t)b * K + ch]);
    float q = rintf(__fdiv_rn(to_f32(k_lat[e]), s));
    q = fminf(fmaxf(q, -127.f), 127.f);
    k_cache[k_elem(lay, kv, b, start + t, c, 1)] = (int8_t)(int)q;
  }
}

// ---- V int4 group quantiser: one warp per (b, t, group of 32 channels).
template <typename LT>
__global__ void __launch_bounds__(256) v_quant_kernel(const starkv_layout lay, const LT* __restrict__ v_lat, int T,
                                                      int start, uint8_t* __restrict__ v_codes,
                                                      __half2* __restrict__ v_params) {
  const int R = lay.v_rank_total;
  const int G = R / 32;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)lay.batch * T * G;
  for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < nwarps;
       w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int g = (int)(w % G);
    const int64_t bt = w / G;
    const int t = (int)(bt % T), b = (int)(bt / T);
    const float x = to_f32(v_lat[bt * R + g * 32 + lane]);
    float mn = x, mx = x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    __half hs = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), 15.0f));
    if (__half2float(hs) == 0.0f) hs = __float2half_rn(1.0f);
    const __half hz = __float2half_rn(mn);
    float q = rintf(__fdiv_rn(__fsub_rn(x, __half2float(hz)), __half2float(hs)));
    q = fminf(fmaxf(q, 0.f), 15.f);
    const uint32_t qi = (uint32_t)(int)q;
    const uint32_t hi = __shfl_down_sync(0xffffffffu, qi, 1);
    const int64_t row = (int64_t)b * lay.capacity + start + t;
    if ((lane & 1) == 0) v_codes[row * (R / 2) + g * 16 + (lane >> 1)] = (uint8_t)(qi | (hi << 4));
    if (lane == 0) v_params[row * G + g] = __halves2half2(hs, hz);
  }
}

// ---- unquantised append: copy latents into the cache rows (same dtype).
template <typename LT>
__global__ void __launch_bounds__(256) copy_append_kernel(const starkv_layout lay, const LT* __restrict__ k_lat,
                                                          const LT* __restrict__ v_lat, int T, int start,
                                                          LT* __restrict__ k_cache, LT* __restrict__ v_cache) {
  const int K = lay.k_rank_total, R = lay.v_rank_total;
  const int64_t nk = (int64_t)lay.batch * T * K;
  const int64_t nv = (int64_t)lay.batch * T * R;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nk + nv;
       e += (int64_t)gridDim.x * blockDim.x) {
    if (e < nk) {
      const int ch = (int)(e % K);
      const int64_t bt = e / K;
      const int t = (int)(bt % T), b = (int)(bt / T);
      int kv = 0;
      while (kv + 1 < lay.num_kv_heads && lay.k_col[kv + 1] <= ch) ++kv;
      const int c = ch - lay.k_col[kv];
      k_cache[k_elem(lay, kv, b, start + t, c, (int)sizeof(LT))] = k_lat[e];
    } else {
      const int64_t f = e - nk;
      const int ch = (int)(f % R);
      const int64_t bt = f / R;
      const int t = (int)(bt % T), b = (int)(bt / T);
      v_cache[((int64_t)b * lay.capacity + start + t) * R + ch] = v_lat[f];
    }
  }
}

}  // namespace starkv

namespace starkv {

// ---- fused latent projection + quantise-append of one decode token per sequence
// (the reference's k_proj.VS / v_proj.VS GEMVs, headwise.py:86-96, followed by the
// cache append, headwise.py:99 / quant.py:107-127).  Channel space: the K latents
// (sum r_h, heads concatenated) then the V latents (R).  One CTA per chunk of 32
// channels (V chunks are the quantiser's groups of 32); its 8 warps split the
// hidden dimension: for every channel of the chunk a warp reads its share of the
// VS row, 16 bytes a lane (coalesced), dots it with every sequence's hidden state
// (staged in shared memory; grid.y = passes of 8 sequences) and reduces with
// shuffles; warp 0 adds the 8 partial sums, rounds to the latent type (the
// reference's projection output) and quantises exactly as the append kernels do;
// k_out / v_out optionally receive the rounded latents.
constexpr int kPaWarps = 8;
template <typename LT>
__host__ __device__ constexpr int kPaSeqOf() { return 8; }

template <typename LT, bool QUANT>
__global__ void __launch_bounds__(kPaWarps * 32) project_append_kernel(
    const starkv_layout lay, const LT* __restrict__ hidden, int H, const LT* __restrict__ vs_k,
    const LT* __restrict__ vs_v, int slot, void* __restrict__ k_cache, const __half* __restrict__ k_scales,
    void* __restrict__ v_cache, __half2* __restrict__ v_params, LT* __restrict__ k_out, LT* __restrict__ v_out) {
  extern __shared__ __align__(16) uint8_t pa_smem[];
  LT* hs = reinterpret_cast<LT*>(pa_smem);                      // [PS][H]
  constexpr int PS = kPaSeqOf<LT>();                            // sequences per pass
  __shared__ float red[kPaWarps][32][PS];                       // per-warp partial dots
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = lay.k_rank_total, R = lay.v_rank_total;
  const int kchunks = (K + 31) / 32;
  const int chunk = blockIdx.x;
  const bool isk = chunk < kchunks;
  const int c0 = isk ? chunk * 32 : (chunk - kchunks) * 32;
  const int nc = isk ? min(32, K - c0) : 32;
  constexpr int VEC = 16 / (int)sizeof(LT);                     // elements per 16-byte load
  if (threadIdx.x < nc)                                         // the chunk's VS rows into L2 (their loads below are serial)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((isk ? vs_k : vs_v) + (int64_t)(c0 + threadIdx.x) * H),
                 "r"((uint32_t)(H * sizeof(LT))) : "memory");
  {
    const int b0 = blockIdx.y * PS;
    const int nb = min(PS, lay.batch - b0);
    __syncthreads();
    for (int e = threadIdx.x * VEC; e < nb * H; e += blockDim.x * VEC)
      *reinterpret_cast<uint4*>(hs + e) = *reinterpret_cast<const uint4*>(hidden + (int64_t)b0 * H + e);
    __syncthreads();
    for (int c = 0; c < nc; c += 4) {                           // 4 channels at a time: their loads in flight together
      const LT* row = (isk ? vs_k : vs_v) + (int64_t)(c0 + c) * H;
      float acc[4][PS];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int s = 0; s < PS; ++s) acc[j][s] = 0.f;
#pragma unroll 2
      for (int k = (warp * 32 + lane) * VEC; k < H; k += kPaWarps * 32 * VEC) {
        uint4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = *reinterpret_cast<const uint4*>(row + (int64_t)j * H + k);
        float wf[4][VEC];                                       // converted once, used for every sequence
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < VEC; ++e) wf[j][e] = to_f32(reinterpret_cast<const LT*>(&w[j])[e]);
#pragma unroll
        for (int s = 0; s < PS; ++s)
          if (s < nb) {
            const uint4 x = *reinterpret_cast<const uint4*>(hs + s * H + k);
            const LT* xv = reinterpret_cast<const LT*>(&x);
            float2 a01 = make_float2(acc[0][s], acc[1][s]), a23 = make_float2(acc[2][s], acc[3][s]);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {                     // two channels per packed fp32x2 FMA
              const float xf = to_f32(xv[e]);
              a01 = __ffma2_rn(make_float2(xf, xf), make_float2(wf[0][e], wf[1][e]), a01);
              a23 = __ffma2_rn(make_float2(xf, xf), make_float2(wf[2][e], wf[3][e]), a23);
            }
            acc[0][s] = a01.x;
            acc[1][s] = a01.y;
            acc[2][s] = a23.x;
            acc[3][s] = a23.y;
          }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int s = 0; s < PS; ++s) {
          float a = acc[j][s];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
          if (lane == 0) red[warp][c + j][s] = a;
        }
    }
    __syncthreads();
    if (warp != 0) return;                                      // no barrier follows
    float mine[PS];                                             // lane = channel c0 + lane: its latent per sequence
#pragma unroll
    for (int s = 0; s < PS; ++s) {
      float a = 0.f;
      if (lane < nc)
#pragma unroll
        for (int w = 0; w < kPaWarps; ++w) a += red[w][lane][s];
      mine[s] = a;
    }
    // round to the latent type, then store / quantise (lane = channel c0 + lane)
    for (int s = 0; s < nb; ++s) {
      const int b = b0 + s;
      const LT lat = from_f32<LT>(mine[s]);
      const float x = to_f32(lat);
      if (isk) {
        if (lane < nc) {
          const int ch = c0 + lane;
          int kv = 0;
          while (kv + 1 < lay.num_kv_heads && lay.k_col[kv + 1] <= ch) ++kv;
          const int c = ch - lay.k_col[kv];
          const int64_t dst = k_elem(lay, kv, b, slot, c, QUANT ? 1 : (int)sizeof(LT));
          if (k_out) k_out[(int64_t)b * K + ch] = lat;
          if constexpr (QUANT) {
            const float sc = __half2float(k_scales[(int64_t)b * K + ch]);
            float q = rintf(__fdiv_rn(x, sc));
            q = fminf(fmaxf(q, -127.f), 127.f);
            reinterpret_cast<int8_t*>(k_cache)[dst] = (int8_t)(int)q;
          } else {
            reinterpret_cast<LT*>(k_cache)[dst] = lat;
          }
        }
      } else {
        const int64_t rowi = (int64_t)b * lay.capacity + slot;
        if (v_out) v_out[(int64_t)b * R + c0 + lane] = lat;
        if constexpr (QUANT) {
          float mn = x, mx = x;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          }
          __half hsc = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), 15.0f));
          if (__half2float(hsc) == 0.0f) hsc = __float2half_rn(1.0f);
          const __half hz = __float2half_rn(mn);
          float q = rintf(__fdiv_rn(__fsub_rn(x, __half2float(hz)), __half2float(hsc)));
          q = fminf(fmaxf(q, 0.f), 15.f);
          const uint32_t qi = (uint32_t)(int)q;
          const uint32_t hi = __shfl_down_sync(0xffffffffu, qi, 1);
          if ((lane & 1) == 0)
            reinterpret_cast<uint8_t*>(v_cache)[rowi * (R / 2) + c0 / 2 + (lane >> 1)] = (uint8_t)(qi | (hi << 4));
          if (lane == 0) v_params[rowi * (R / 32) + c0 / 32] = __halves2half2(hsc, hz);
        } else {
          reinterpret_cast<LT*>(v_cache)[rowi * R + c0 + lane] = lat;
        }
      }
    }
  }
}

// ---- split format of the reference's quantiser interface
// (quantize_r_split_int8_int4_packed, called at LlamaLoRaAttention_headwise_quant.py:107-117):
// per row, the first split_r values as int8 with one symmetric fp16 scale
// (absmax / 127), the rest as signed int4 with one symmetric fp16 scale
// (absmax / 7), stored as nibble q + 8, even rank in the low nibble.  One warp per row.
template <typename LT>
__global__ void __launch_bounds__(256) split_quant_kernel(const LT* __restrict__ x, int64_t rows, int r, int split_r,
                                                          int8_t* __restrict__ up, __half* __restrict__ s_up,
                                                          uint8_t* __restrict__ lo, __half* __restrict__ s_lo) {
  const int lane = threadIdx.x & 31;
  const int r4 = r - split_r;
  for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < rows;
       w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const LT* xr = x + w * r;
    float au = 0.f, al = 0.f;
    for (int c = lane; c < r; c += 32) {
      const float v = fabsf(to_f32(xr[c]));
      if (c < split_r) au = fmaxf(au, v); else al = fmaxf(al, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      au = fmaxf(au, __shfl_xor_sync(0xffffffffu, au, o));
      al = fmaxf(al, __shfl_xor_sync(0xffffffffu, al, o));
    }
    __half hu = __float2half_rn(__fdiv_rn(au, 127.0f)), hl = __float2half_rn(__fdiv_rn(al, 7.0f));
    if (__half2float(hu) == 0.0f) hu = __float2half_rn(1.0f);
    if (__half2float(hl) == 0.0f) hl = __float2half_rn(1.0f);
    if (lane == 0) {
      if (split_r > 0) s_up[w] = hu;
      if (r4 > 0) s_lo[w] = hl;
    }
    const float su = __half2float(hu), sl = __half2float(hl);
    for (int c = lane; c < split_r; c += 32) {
      const float q = fminf(fmaxf(rintf(__fdiv_rn(to_f32(xr[c]), su)), -127.f), 127.f);
      up[w * split_r + c] = (int8_t)(int)q;
    }
    for (int c2 = lane; c2 < (r4 + 1) / 2; c2 += 32) {
      uint32_t byte = 0;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = 2 * c2 + k;
        if (c < r4) {
          const float q = fminf(fmaxf(rintf(__fdiv_rn(to_f32(xr[split_r + c]), sl)), -8.f), 7.f);
          byte |= ((uint32_t)((int)q + 8) & 0xFu) << (4 * k);
        }
      }
      lo[w * ((r4 + 1) / 2) + c2] = (uint8_t)byte;
    }
  }
}

}  // namespace starkv
