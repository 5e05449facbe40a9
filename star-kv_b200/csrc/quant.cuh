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
// grid (Hkv, B), block 256.  k_lat: (B, T, k_rank_total) latent dtype.
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
    k_scales[(int64_t)b * K + lay.k_col[kv] + c] = h;
    sc[c] = __half2float(h);
  }
  __syncthreads();
  int8_t* dst = k_cache + lay.k_offset[kv] + (int64_t)b * lay.k_batch_stride[kv];
  for (int64_t e = threadIdx.x; e < (int64_t)T * r; e += blockDim.x) {
    const int t = (int)(e / r), c = (int)(e % r);
    float q = rintf(__fdiv_rn(to_f32(src[(int64_t)t * K + c]), sc[c]));
    q = fminf(fmaxf(q, -127.f), 127.f);
    dst[(int64_t)t * r + c] = (int8_t)(int)q;
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
    const int r = lay.k_rank[kv];
    const float s = __half2float(k_scales[(int64_t)b * K + ch]);
    float q = rintf(__fdiv_rn(to_f32(k_lat[e]), s));
    q = fminf(fmaxf(q, -127.f), 127.f);
    k_cache[lay.k_offset[kv] + (int64_t)b * lay.k_batch_stride[kv] + (int64_t)(start + t) * r + c] = (int8_t)(int)q;
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
      const int c = ch - lay.k_col[kv], r = lay.k_rank[kv];
      k_cache[lay.k_offset[kv] + (int64_t)b * lay.k_batch_stride[kv] + (int64_t)(start + t) * r + c] = k_lat[e];
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
