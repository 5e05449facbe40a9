// v_latent.cuh — V path of the decode step: softmax weights x dequantised V
// latents, in latent space (the reorder branch of
// LlamaLoRaAttention_headwise.py:126-133 / model.py:482-487; bx_quant._bx_fwd,
// bx_quant.py:38-114), then the V up-projection once per head.
//
// int4 V with per-token groups of 32 (scale s, zero z): for a head with weights p_l,
//   sum_l p_l x_hat[l, c] = sum_l (p_l s_lg) q_lc + sum_l p_l z_lg      (g = c / 32)
// so each token costs one multiply per (head, group) plus one FMA per (head, channel),
// and the zero point is one accumulator per (head, group).
#pragma once
#include "common.cuh"

namespace starkv {

struct VParams {
  starkv_layout lay;
  const float* logits;   // (B, Hq, T) log2-domain logits (decode) ...
  const float2* stats;   // (B, Hq, nsplit_k) split (max, sum exp2)
  const float* probs;    // ... or (B, Hq, T) probabilities (bx mode) when non-null
  const void* v_cache;
  const __half2* v_params;
  float* partial;        // decode: (B, Hq, nsplit, rv_max); bx mode: (B, Hq, R)
  int T, nsplit, nsplit_k, tps, rv_max;
};

constexpr int kVThreads = 256;
constexpr int kVChunk = 64;
constexpr int kVMaxHeads = 8;

__host__ __device__ inline size_t v_smem_bytes(int heads) {
  return (size_t)kVMaxHeads * 2 * sizeof(float) + (size_t)heads * kVChunk * sizeof(float) +
         (size_t)kVThreads * heads * 8 * sizeof(float);
}

// 8 consecutive V latents of one token row as floats.
template <typename LT>
__device__ __forceinline__ void load8(const LT* src, float* x) {
  if constexpr (sizeof(LT) == 4) {
    const float4 a = reinterpret_cast<const float4*>(src)[0], c = reinterpret_cast<const float4*>(src)[1];
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(src);
    const LT* h = reinterpret_cast<const LT*>(&w);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = to_f32(h[k]);
  }
}

// grid (nsplit, num_v_blocks, B), 256 threads.  LT = latent type (unquantised) or uint8_t (int4 codes).
template <typename LT, bool QUANT>
__global__ void __launch_bounds__(kVThreads) v_latent_kernel(const __grid_constant__ VParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const starkv_layout& lay = p.lay;
  const int split = blockIdx.x, blk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int qh0 = lay.v_first_kv[blk] * qpk;
  const int Gv = lay.v_num_kv[blk] * qpk;
  const int r = lay.v_rank[blk], vcol = lay.v_col[blk];
  const int R = lay.v_rank_total;
  const int CG = r >> 3;                 // 8-channel column groups
  const int NS = kVThreads / CG;         // token slots
  const int cg = tid % CG, ts = tid / CG;
  const int t_begin = split * p.tps, t_end = min(p.T, t_begin + p.tps);

  float* s_mx = reinterpret_cast<float*>(smem);           // [8]
  float* s_il = s_mx + kVMaxHeads;                         // [8]
  float* s_p = s_il + kVMaxHeads;                          // [Gv][64]
  float* s_red = s_p + Gv * kVChunk;                       // [NS * CG][Gv][8]

  if (!p.probs) {
    if (warp < Gv) {
      const int qh = qh0 + warp;
      float m = kNegBig, l = 0.f;
      for (int s = lane; s < p.nsplit_k; s += 32) {
        const float2 st = p.stats[((int64_t)b * Hq + qh) * p.nsplit_k + s];
        softmax_merge(m, l, st.x, st.y);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
        softmax_merge(m, l, m2, l2);
      }
      if (lane == 0) { s_mx[warp] = m; s_il[warp] = l > 0.f ? 1.f / l : 0.f; }
    }
  }
  __syncthreads();

  float acc[kVMaxHeads][8];
  float zacc[kVMaxHeads];
#pragma unroll
  for (int g = 0; g < kVMaxHeads; ++g) {
    zacc[g] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[g][k] = 0.f;
  }

  for (int c0 = t_begin; c0 < t_end; c0 += kVChunk) {
    for (int e = tid; e < Gv * kVChunk; e += kVThreads) {
      const int t = e % kVChunk, g = e / kVChunk, l = c0 + t;
      float pv = 0.f;
      if (l < t_end) {
        const int64_t idx = ((int64_t)b * Hq + qh0 + g) * p.T + l;
        pv = p.probs ? p.probs[idx] : exp2f(p.logits[idx] - s_mx[g]) * s_il[g];
      }
      s_p[g * kVChunk + t] = pv;
    }
    __syncthreads();
    if (ts < NS) {
      const int nt = min(kVChunk, t_end - c0);
      for (int t = ts; t < nt; t += NS) {
        const int64_t row = (int64_t)b * lay.capacity + c0 + t;
        float x[8];
        float s = 1.f, z = 0.f;
        if constexpr (QUANT) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(p.v_cache) +
                                                                row * (R / 2) + vcol / 2 + cg * 4);
#pragma unroll
          for (int k = 0; k < 8; ++k) x[k] = (float)((w >> (4 * k)) & 15u);
          const float2 sz = __half22float2(p.v_params[row * (R / 32) + vcol / 32 + cg / 4]);
          s = sz.x;
          z = sz.y;
        } else {
          load8<LT>(reinterpret_cast<const LT*>(p.v_cache) + row * R + vcol + cg * 8, x);
        }
#pragma unroll
        for (int g = 0; g < kVMaxHeads; ++g) {
          if (g < Gv) {
            const float pv = s_p[g * kVChunk + t];
            const float ps = QUANT ? pv * s : pv;
            if (QUANT) zacc[g] = fmaf(pv, z, zacc[g]);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[g][k] = fmaf(ps, x[k], acc[g][k]);
          }
        }
      }
    }
    __syncthreads();
  }

  // reduce over token slots
  if (ts < NS) {
#pragma unroll
    for (int g = 0; g < kVMaxHeads; ++g)
      if (g < Gv)
#pragma unroll
        for (int k = 0; k < 8; ++k) s_red[((size_t)tid * Gv + g) * 8 + k] = acc[g][k] + zacc[g];
  }
  __syncthreads();
  for (int e = tid; e < Gv * r; e += kVThreads) {
    const int g = e / r, c = e % r;
    const int ccg = c >> 3, k = c & 7;
    float sum = 0.f;
    for (int s = 0; s < NS; ++s) sum += s_red[((size_t)(s * CG + ccg) * Gv + g) * 8 + k];
    const int qh = qh0 + g;
    if (p.probs)
      p.partial[((int64_t)b * Hq + qh) * R + vcol + c] = sum;
    else
      p.partial[(((int64_t)b * Hq + qh) * p.nsplit + split) * p.rv_max + c] = sum;
  }
}

// Merge the split partials and apply the V up-projection once per head:
//   out[b, h, d] = sum_c (sum_s partial[b, h, s, c]) * U_v[kv * 128 + d, vcol + c]
// grid (Hq, B), 128 threads.
struct CombineParams {
  starkv_layout lay;
  const float* partial;
  const void* v_u;
  void* out;
  int w_dtype, out_dtype, nsplit, rv_max;
};

__global__ void __launch_bounds__(128) combine_kernel(const __grid_constant__ CombineParams p) {
  __shared__ float o_lat[256];
  const starkv_layout& lay = p.lay;
  const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads, kv = qh / qpk;
  int blk = 0;
  while (blk + 1 < lay.num_v_blocks && lay.v_first_kv[blk + 1] <= kv) ++blk;
  const int r = lay.v_rank[blk], vcol = lay.v_col[blk], R = lay.v_rank_total;
  for (int c = tid; c < r; c += 128) {
    float s = 0.f;
    const float* src = p.partial + ((int64_t)b * Hq + qh) * p.nsplit * p.rv_max + c;
    for (int k = 0; k < p.nsplit; ++k) s += src[(int64_t)k * p.rv_max];
    o_lat[c] = s;
  }
  __syncthreads();
  const int64_t urow = ((int64_t)kv * 128 + tid) * R + vcol;
  float acc = 0.f;
  for (int c = 0; c < r; ++c) acc = fmaf(o_lat[c], load_as_f32(p.v_u, p.w_dtype, urow + c), acc);
  store_from_f32(p.out, p.out_dtype, ((int64_t)b * Hq + qh) * 128 + tid, acc);
}

}  // namespace starkv
