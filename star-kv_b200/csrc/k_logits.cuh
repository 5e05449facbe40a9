// k_logits.cuh — fused K path of the decode step on the sm_100a tensor cores.
//
// Replaces abx_rope_batched._abx_fwd (abx_rope_batched.py:60-132) and the eager
// K reconstruction + RoPE + q.k of LlamaLoRaAttention_headwise.py:107-110.
//
// For one query head h (KV head kv, rank r) and cached token l:
//     logit_l = q . RoPE_l(x_l @ U^T),   x_l = dequant(X_k[b, kv, l, :]) (r),  U (128 x r)
// With the half-split RoPE (rotate_half) and c_i = cos(l w_i), s_i = sin(l w_i):
//     q . RoPE_l(k) = sum_i c_i (q_i k_i + q_{i+64} k_{i+64}) + s_i (q_{i+64} k_i - q_i k_{i+64})
// so with the per-head r x 128 matrix W = [P | Q],
//     P[c, i] = sc_c (q_i U[i, c] + q_{i+64} U[i+64, c]),
//     Q[c, i] = sc_c (q_{i+64} U[i, c] - q_i U[i+64, c])        (sc_c = K channel scale)
// the whole K path is one GEMM  D = X_codes (tokens x r) @ W (r x 128)  on the
// tensor cores followed by  logit_l = sum_i c_i D[l, i] + s_i D[l, 64 + i]  in the
// TMEM drain.  The query is folded into W once per CTA, so neither the keys
// nor the rotated keys are ever materialised.
//
// CTA = (sequence split, group of G query heads, sequence b); 128 threads, one
// token row of a 128-token tile per thread.  Per (tile, head) "job":
//   bulk copy (global -> smem staging ring, S stages, issued S-1 jobs ahead)
//   -> convert the codes to fp16 into the canonical no-swizzle A layout
//   -> one thread issues r/16 tcgen05.mma (M=128, N=128, K=16) into TMEM
//      (two accumulators, ping-pong: the MMA of job j runs during the drain of j-1)
//   -> drain: tcgen05.ld, RoPE-weighted reduction, mask, logits to global and an
//      online (max, sum exp2) per head for the split-softmax merge.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace starkv {

struct KParams {
  starkv_layout lay;
  const void* q;
  const void* k_u;
  const void* k_cache;
  const __half* k_scales;
  const float2* rope;   // (>= T, 64) (cos, sin) of fl(l * inv_freq_i)
  const float* mask;    // (B, T) additive or null
  float* logits;        // (B, Hq, T)
  float2* stats;        // (B, Hq, nsplit) (max, sum exp2) or null
  int* err;
  int q_dtype, w_dtype;
  int T, nsplit, tps;   // tokens, splits, tokens per split (multiple of 128)
  int G, S, rmax;       // heads per CTA, staging stages, max rank (smem strides)
  float out_scale;      // multiplier of q.k (scaling * log2 e for decode)
  float mask_scale;     // multiplier of the mask (log2 e for decode)
};

constexpr int kKThreads = 128;
constexpr int kKHeader = 2048;  // bytes of barriers / scratch at the start of dynamic smem

__host__ __device__ inline size_t k_smem_bytes(int G, int S, int rmax, int xbytes) {
  return (size_t)kKHeader + (size_t)G * rmax * 256 + (size_t)2 * rmax * 256 + (size_t)S * 128 * rmax * xbytes;
}

// 8 consecutive latent elements -> 8 fp16 (exact for int8 codes and fp16/bf16 values).
template <typename XT>
__device__ __forceinline__ uint4 cvt8_f16(const uint8_t* src);

template <>
__device__ __forceinline__ uint4 cvt8_f16<int8_t>(const uint8_t* src) {
  const uint2 w = *reinterpret_cast<const uint2*>(src);
  // int8 x -> (x + 128) as a byte; 0x64XX as fp16 is 1024 + XX; subtract 1152.
  const uint32_t a = w.x ^ 0x80808080u, b = w.y ^ 0x80808080u;
  uint4 o;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
  uint32_t t;
  t = __byte_perm(a, 0x64646464u, 0x5140); { __half2 h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.x = *reinterpret_cast<uint32_t*>(&h); }
  t = __byte_perm(a, 0x64646464u, 0x7362); { __half2 h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.y = *reinterpret_cast<uint32_t*>(&h); }
  t = __byte_perm(b, 0x64646464u, 0x5140); { __half2 h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.z = *reinterpret_cast<uint32_t*>(&h); }
  t = __byte_perm(b, 0x64646464u, 0x7362); { __half2 h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.w = *reinterpret_cast<uint32_t*>(&h); }
  return o;
}

template <>
__device__ __forceinline__ uint4 cvt8_f16<__half>(const uint8_t* src) {
  return *reinterpret_cast<const uint4*>(src);
}

template <>
__device__ __forceinline__ uint4 cvt8_f16<__nv_bfloat16>(const uint8_t* src) {
  const uint4 w = *reinterpret_cast<const uint4*>(src);
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t out[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float lo = __uint_as_float(in[k] << 16), hi = __uint_as_float(in[k] & 0xFFFF0000u);
    __half2 h = __floats2half2_rn(lo, hi);
    out[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <>
__device__ __forceinline__ uint4 cvt8_f16<float>(const uint8_t* src) {
  const float4 a = reinterpret_cast<const float4*>(src)[0];
  const float4 b = reinterpret_cast<const float4*>(src)[1];
  __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
  __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
  return make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                    *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
}

template <typename XT, bool QUANT>
__global__ void __launch_bounds__(kKThreads, 1) k_logits_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int split = blockIdx.x, grp = blockIdx.y, b = blockIdx.z;
  const starkv_layout& lay = p.lay;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int G = p.G, S = p.S, rmax = p.rmax;
  const int t_begin = split * p.tps;
  const int t_end = min(p.T, t_begin + p.tps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + 127) / 128 : 0;
  const int J = ntiles * G;

  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);   // [8]
  uint64_t* mma_bar = full_bar + 8;                          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 2);
  float* s_red = reinterpret_cast<float*>(smem + 256);       // [8]
  float* s_q = reinterpret_cast<float*>(smem + 512);         // [128]
  float* s_epi = reinterpret_cast<float*>(smem + 1024);      // [4] per-head drain multiplier
  uint8_t* Bsm = smem + kKHeader;
  uint8_t* Asm = Bsm + (size_t)G * rmax * 256;
  uint8_t* Ssm = Asm + (size_t)2 * rmax * 256;
  const uint32_t stage_bytes = 128u * rmax * sizeof(XT);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(full_bar + s, 1);
    mbar_init(mma_bar + 0, 1);
    mbar_init(mma_bar + 1, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Per-job geometry.
  auto job_head = [&](int j, int& qh, int& kv, int& r) {
    const int g = j % G;
    qh = grp * G + g;
    kv = qh / qpk;
    r = lay.k_rank[kv];
  };
  auto issue_copy = [&](int j) {
    int qh, kv, r;
    job_head(j, qh, kv, r);
    const int t0 = t_begin + (j / G) * 128;
    const int n = min(128, t_end - t0);
    const uint32_t bytes = (uint32_t)(n * r * (int)sizeof(XT));
    const XT* src = reinterpret_cast<const XT*>(p.k_cache) + lay.k_offset[kv] +
                    (int64_t)b * lay.k_batch_stride[kv] + (int64_t)t0 * r;
    uint64_t* bar = full_bar + (j % S);
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(Ssm + (size_t)(j % S) * stage_bytes, src, bytes, bar);
  };

  if (tid == 0)
    for (int j = 0; j < min(S - 1, J); ++j) issue_copy(j);

  // ---- build W_g = [P | Q] (fp16, canonical K-major layout) for each head of the group.
  for (int g = 0; g < G; ++g) {
    const int qh = grp * G + g, kv = qh / qpk, r = lay.k_rank[kv];
    s_q[tid] = load_as_f32(p.q, p.q_dtype, ((int64_t)b * Hq + qh) * 128 + tid);
    __syncthreads();
    float* scr = reinterpret_cast<float*>(Asm);  // [r][128] fp32 scratch (fits the A buffers)
    const int64_t ubase = (int64_t)128 * lay.k_col[kv];
    float amax = 0.f;
    for (int e = tid; e < r * 64; e += kKThreads) {
      const int c = e >> 6, i = e & 63;
      const float u1 = load_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)i * r + c);
      const float u2 = load_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)(i + 64) * r + c);
      const float sc = QUANT ? __half2float(p.k_scales[(int64_t)b * lay.k_rank_total + lay.k_col[kv] + c]) : 1.f;
      const float qa = s_q[i], qb = s_q[i + 64];
      const float P = sc * (qa * u1 + qb * u2);
      const float Q = sc * (qb * u1 - qa * u2);
      scr[c * 128 + i] = P;
      scr[c * 128 + 64 + i] = Q;
      amax = fmaxf(amax, fmaxf(fabsf(P), fabsf(Q)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((tid & 31) == 0) s_red[warp] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    // Power-of-two normalisation: entries of W land in [2^13, 2^14] at the top,
    // keeping fp16's full precision; undone exactly in the drain.
    const float eta = amax > 0.f ? exp2f(ceilf(log2f(amax)) - 14.f) : 1.f;
    const float inv_eta = 1.f / eta;
    if (tid == 0) s_epi[g] = eta * p.out_scale;
    uint8_t* Bg = Bsm + (size_t)g * rmax * 256;
    const int nc = r >> 3;
    for (int e = tid; e < 128 * nc; e += kKThreads) {
      const int n = e & 127, kc = e >> 7;
      __align__(16) __half h[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) h[k] = __float2half_rn(scr[(kc * 8 + k) * 128 + n] * inv_eta);
      *reinterpret_cast<uint4*>(Bg + (n >> 3) * (r * 16) + kc * 128 + (n & 7) * 16) = *reinterpret_cast<uint4*>(h);
    }
    __syncthreads();
  }

  constexpr uint32_t IDESC = idesc_f16_f32(128, 128);
  float m_run[4] = {kNegBig, kNegBig, kNegBig, kNegBig};
  float l_run[4] = {0.f, 0.f, 0.f, 0.f};
  float2 cs[64];
  int last_mma = -1;
  bool failed = false;

  for (int j = 0; j <= J; ++j) {
    int fail = 0;
    if (j < J) {
      // ---- wait for job j's codes, convert into A[j & 1]
      if (!mbar_wait(full_bar + (j % S), (uint32_t)((j / S) & 1))) {
        record_error(p.err, kDevWaitCopy);
        fail = 1;
      } else {
        int qh, kv, r;
        job_head(j, qh, kv, r);
        const int t0 = t_begin + (j / G) * 128;
        const int n = min(128, t_end - t0);
        const int nc = r >> 3;
        const uint8_t* stg = Ssm + (size_t)(j % S) * stage_bytes;
        uint8_t* A = Asm + (size_t)(j & 1) * rmax * 256;
        for (int e = tid; e < 128 * nc; e += kKThreads) {
          const int ri = e & 7, rest = e >> 3;
          const int c = rest % nc, rg = rest / nc;
          const int row = rg * 8 + ri;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (row < n) v = cvt8_f16<XT>(stg + ((size_t)row * r + c * 8) * sizeof(XT));
          *reinterpret_cast<uint4*>(A + rg * (r * 16) + c * 128 + ri * 16) = v;
        }
      }
      fence_proxy_async_smem();
    }
    tc_fence_before();
    if (__syncthreads_or(fail)) {
      failed = true;
      break;
    }
    if (tid == 0) {
      if (j + S - 1 < J) issue_copy(j + S - 1);
      if (j < J) {
        tc_fence_after();
        int qh, kv, r;
        job_head(j, qh, kv, r);
        const uint32_t a0 = smem_u32(Asm + (size_t)(j & 1) * rmax * 256);
        const uint32_t b0 = smem_u32(Bsm + (size_t)(j % G) * rmax * 256);
        const uint32_t sbo = (uint32_t)r * 16u;
        const uint32_t d = tmem + (uint32_t)(j & 1) * 128u;
        for (int k = 0; k < r / 16; ++k)
          mma_f16_ss(d, smem_desc(a0 + k * 256, 128, sbo), smem_desc(b0 + k * 256, 128, sbo), IDESC, k > 0 ? 1u : 0u);
        mma_commit(mma_bar + (j & 1));
        last_mma = j;
      }
    }
    if (j >= 1) {
      // ---- drain job j-1
      const int jj = j - 1, buf = jj & 1, g = jj % G;
      const int tile = jj / G;
      const int l = t_begin + tile * 128 + tid;
      const bool valid = l < t_end;
      if (g == 0) {
        const float4* row = reinterpret_cast<const float4*>(p.rope + (int64_t)(valid ? l : t_begin) * 64);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float4 v = __ldg(row + k);
          cs[2 * k] = make_float2(v.x, v.y);
          cs[2 * k + 1] = make_float2(v.z, v.w);
        }
      }
      const bool ok = mbar_wait(mma_bar + buf, (uint32_t)((jj >> 1) & 1));
      if (!ok) record_error(p.err, kDevWaitMma);
      tc_fence_after();
      if (ok) {
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)buf * 128u;
        float v[32];
        float acc = 0.f;
        tmem_ld32(taddr + 0, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc = fmaf(cs[i].x, v[i], acc);
        tmem_ld32(taddr + 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc = fmaf(cs[32 + i].x, v[i], acc);
        tmem_ld32(taddr + 64, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc = fmaf(cs[i].y, v[i], acc);
        tmem_ld32(taddr + 96, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc = fmaf(cs[32 + i].y, v[i], acc);
        if (valid) {
          const int qh = grp * G + g;
          float val = acc * s_epi[g];
          if (p.mask) val = fmaf(p.mask[(int64_t)b * p.T + l], p.mask_scale, val);
          p.logits[((int64_t)b * Hq + qh) * p.T + l] = val;
#pragma unroll
          for (int gg = 0; gg < 4; ++gg)
            if (gg == g) softmax_merge(m_run[gg], l_run[gg], val, 1.f);
        }
      }
      tc_fence_before();
    }
  }

  // ---- split statistics: (max, sum exp2(logit - max)) per head over this split.
  if (!failed && p.stats) {
    float* s_m = s_red;          // reuse: [4 warps]
    float* s_l = s_red + 4;
    for (int g = 0; g < G; ++g) {
      float m = kNegBig, l = 0.f;
#pragma unroll
      for (int gg = 0; gg < 4; ++gg)
        if (gg == g) { m = m_run[gg]; l = l_run[gg]; }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
        softmax_merge(m, l, m2, l2);
      }
      __syncthreads();
      if ((tid & 31) == 0) { s_m[warp] = m; s_l[warp] = l; }
      __syncthreads();
      if (tid == 0) {
        float M = s_m[0], Lsum = s_l[0];
        for (int w = 1; w < 4; ++w) softmax_merge(M, Lsum, s_m[w], s_l[w]);
        p.stats[((int64_t)b * Hq + grp * G + g) * p.nsplit + split] = make_float2(M, Lsum);
      }
    }
  }

  // ---- teardown: nothing of ours may still be writing TMEM / smem.
  if (failed && tid == 0) {
    if (last_mma >= 0) (void)mbar_wait(mma_bar + (last_mma & 1), (uint32_t)((last_mma >> 1) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// RoPE table: rope[l][i] = (cos, sin)(fl(l * inv_freq[i])) — the fp32 angle HF's
// LlamaRotaryEmbedding forms (inv_freq @ position_ids in fp32), then CUDA's
// full-precision sincosf.
__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int t0, int n, float2* __restrict__ rope) {
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= (int64_t)n * 64) return;
  const int l = t0 + (int)(e >> 6), i = (int)(e & 63);
  const float ang = __fmul_rn((float)l, inv_freq[i]);
  float s, c;
  sincosf(ang, &s, &c);
  rope[(int64_t)l * 64 + i] = make_float2(c, s);
}

}  // namespace starkv
