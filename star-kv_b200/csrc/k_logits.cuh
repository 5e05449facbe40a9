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
// CTA = (sequence split, group of G query heads, sequence b).  A "job" is one
// (128-token tile, head) pair; jobs flow through three warp-specialised roles
// that hand off through mbarriers, so copy, conversion, MMA and drain of
// different jobs overlap:
//   converter warps (4): 16-byte cp.async of each job's codes into an S-stage
//                    ring (rows padded to an odd number of 16-byte chunks so
//                    that row reads are bank-conflict free), issued S-1 jobs
//                    ahead; then codes -> fp16 into the canonical no-swizzle
//                    K-major A layout (NA buffers);
//   MMA warp (1)   : one thread issues r/16 tcgen05.mma (M=128, N=128, K=16)
//                    into one of ND TMEM accumulators and commits;
//   drain warps (4): tcgen05.ld of the accumulator row of their token, the
//                    RoPE-weighted reduction, mask, logits to global, and an
//                    online (max, sum exp2) per head for the split-softmax merge.
//
// RoPE angles: each drain thread owns one token row of every tile; it starts
// from cos/sin of l*w_i for its first token and advances by the exact rotation
// through 128*w_i per tile (fp32, 4 FMA per frequency per tile, shared by the
// G heads).  The angles are the exact l*w_i; the reference's fp32 product
// fl(l*w_i) differs from them by at most half an ulp of the angle.
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
  const float* inv_freq;  // (64,) fp32 RoPE inverse frequencies
  const float* mask;      // (B, T) additive or null
  float* logits;          // (B, Hq, T)
  float2* stats;          // (B, Hq, nsplit) (max, sum exp2) or null
  int* err;
  int q_dtype, w_dtype;
  int T, nsplit, tps;     // tokens, splits, tokens per split (multiple of 128)
  int G, rmax, bsum;      // heads per CTA, max rank, max per-group rank sum (W matrices in smem)
  float out_scale;        // multiplier of q.k (scaling * log2 e for decode)
  float mask_scale;       // multiplier of the mask (log2 e for decode)
  long long* trace;       // optional per-job clock64 timeline of CTAs (0, 0, b < 2); null = off
  int trace_jobs;         // jobs recorded per traced CTA
};

// Per-job timeline fields (clock64 of the SM).
enum KTrace {
  kTrConvBegin = 0, kTrConvLanded, kTrConvAEmpty, kTrConvCvt, kTrConvDone, kTrMmaIssue, kTrDrainWait, kTrDrainGot,
  kTrDrainDone, kTrFields = 10
};

constexpr int kKConvWarps = 4, kKDrainWarps = 4;
constexpr int kKMmaWarp = kKConvWarps + kKDrainWarps;              // warp 8
constexpr int kKThreads = 32 * (kKMmaWarp + 1);
constexpr int kKWorkers = 32 * (kKConvWarps + kKDrainWarps);     // threads that build W
constexpr int kKStages = 4;      // staging ring depth (jobs) for 1- and 2-byte latents
constexpr int kKNumA = 2;        // converted A buffers
constexpr int kKNumD = 4;        // TMEM accumulators (4 x 128 columns)
constexpr int kKHeader = 4096;   // barriers / scratch at the start of dynamic smem

// fp32 latents (4x the bytes of int8 codes) use a two-slot ring.
__host__ __device__ constexpr int k_stages(int xbytes) { return xbytes == 4 ? 2 : kKStages; }

// Staging row pitch in 16-byte units: the row's chunks rounded up to an odd count.
__host__ __device__ inline int k_pitch16(int r, int xbytes) { return ((r * xbytes) >> 4) | 1; }

__host__ __device__ inline size_t k_smem_bytes(int bsum, int rmax, int xbytes) {
  return (size_t)kKHeader + (size_t)bsum * 256 + (size_t)kKNumA * rmax * 256 +
         (size_t)k_stages(xbytes) * 128 * k_pitch16(rmax, xbytes) * 16;
}

// 8 int8 codes -> 8 fp16 (exact): x -> (x + 128) as a byte; 0x64XX as fp16 is
// 1024 + XX; subtract 1152.
__device__ __forceinline__ uint4 cvt8_i8(uint32_t lo, uint32_t hi) {
  const uint32_t a = lo ^ 0x80808080u, b = hi ^ 0x80808080u;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
  uint4 o;
  uint32_t t;
  __half2 h;
  t = __byte_perm(a, 0x64646464u, 0x5140); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.x = *reinterpret_cast<uint32_t*>(&h);
  t = __byte_perm(a, 0x64646464u, 0x7362); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.y = *reinterpret_cast<uint32_t*>(&h);
  t = __byte_perm(b, 0x64646464u, 0x5140); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.z = *reinterpret_cast<uint32_t*>(&h);
  t = __byte_perm(b, 0x64646464u, 0x7362); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o.w = *reinterpret_cast<uint32_t*>(&h);
  return o;
}

// Convert one 16-byte staging chunk into fp16 A chunks of `arow`; kc0 indexes
// 8-element A chunks (fp32: half A chunks).
template <typename XT>
__device__ __forceinline__ void cvt_chunk(const uint4 w, uint8_t* arow, int kc0);

template <>
__device__ __forceinline__ void cvt_chunk<int8_t>(const uint4 w, uint8_t* arow, int kc0) {
  *reinterpret_cast<uint4*>(arow + kc0 * 128) = cvt8_i8(w.x, w.y);
  *reinterpret_cast<uint4*>(arow + (kc0 + 1) * 128) = cvt8_i8(w.z, w.w);
}
template <>
__device__ __forceinline__ void cvt_chunk<__half>(const uint4 w, uint8_t* arow, int kc0) {
  *reinterpret_cast<uint4*>(arow + kc0 * 128) = w;
}
template <>
__device__ __forceinline__ void cvt_chunk<__nv_bfloat16>(const uint4 w, uint8_t* arow, int kc0) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t out[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float lo = __uint_as_float(in[k] << 16), hi = __uint_as_float(in[k] & 0xFFFF0000u);
    __half2 h = __floats2half2_rn(lo, hi);
    out[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(arow + kc0 * 128) = make_uint4(out[0], out[1], out[2], out[3]);
}
template <>
__device__ __forceinline__ void cvt_chunk<float>(const uint4 w, uint8_t* arow, int kc0) {
  __half2 h0 = __floats2half2_rn(__uint_as_float(w.x), __uint_as_float(w.y));
  __half2 h1 = __floats2half2_rn(__uint_as_float(w.z), __uint_as_float(w.w));
  *reinterpret_cast<uint2*>(arow + (kc0 >> 1) * 128 + (kc0 & 1) * 8) =
      make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
}

// A-chunk index advance per 16-byte staging chunk.
template <typename XT>
__host__ __device__ constexpr int kc_per_chunk() { return sizeof(XT) == 1 ? 2 : 1; }

// cos/sin of the exact angle l*w (w an fp32 value): the product is exact in
// double; it is reduced by the nearest multiple of 2*pi in double, and the
// fp32 sine/cosine of the reduced angle (|x| <= pi) is taken.
__device__ __forceinline__ void exact_sincos(int l, float w, float& c, float& s) {
  const double a = (double)l * (double)w;
  const double k = rint(a * 0.15915494309189533577);          // a / (2 pi)
  const double red = fma(-k, 6.28318530717958647693, a);
  __sincosf((float)red, &s, &c);
}

template <typename XT, bool QUANT>
__global__ void __launch_bounds__(kKThreads, 1) k_logits_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, grp = blockIdx.y, b = blockIdx.z;
  const starkv_layout& lay = p.lay;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int G = p.G, rmax = p.rmax;
  const int t_begin = split * p.tps;
  const int t_end = min(p.T, t_begin + p.tps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + 127) / 128 : 0;
  const int J = ntiles * G;
  constexpr int XB = (int)sizeof(XT);
  constexpr int STG = k_stages(XB);

  // ---- shared memory carve-up
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* a_full = bars + 0;         // [NA]  4 converter warps wrote A
  uint64_t* a_empty = bars + 2;        // [NA]  MMA done reading A (commit)
  uint64_t* d_full = bars + 4;         // [ND]  accumulator ready (commit)
  uint64_t* d_empty = bars + 8;        // [ND]  4 drain warps done reading
  uint64_t* fin_bar = bars + 12;       //       teardown: every issued MMA retired
  uint64_t* w_ready = bars + 13;       //       the 8 worker warps finished W
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 512);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 516);
  int* s_boff = reinterpret_cast<int*>(smem + 528);           // [4] byte offset of W_g
  float* s_red = reinterpret_cast<float*>(smem + 576);        // [64]
  float* s_epi = reinterpret_cast<float*>(smem + 832);        // [4]
  float2* s_rot = reinterpret_cast<float2*>(smem + 1024);     // [64] rotation by 128 positions
  float* s_q = reinterpret_cast<float*>(smem + 2048);         // [G][128]
  uint8_t* Bsm = smem + kKHeader;
  uint8_t* Asm = Bsm + (size_t)p.bsum * 256;
  uint8_t* Ssm = Asm + (size_t)kKNumA * rmax * 256;
  const uint32_t slot_bytes = 128u * k_pitch16(rmax, XB) * 16u;

  if (tid == 0) {
    for (int k = 0; k < kKNumA; ++k) { mbar_init(a_full + k, kKConvWarps); mbar_init(a_empty + k, 1); }
    for (int k = 0; k < kKNumD; ++k) { mbar_init(d_full + k, 1); mbar_init(d_empty + k, kKDrainWarps); }
    mbar_init(fin_bar, 1);
    mbar_init(w_ready, kKConvWarps + kKDrainWarps);
    *s_abort = 0;
    int off = 0;
    for (int g = 0; g < G; ++g) {
      s_boff[g] = off;
      off += lay.k_rank[(grp * G + g) / qpk] * 256;
    }
    fence_mbar_init();
  }
  if (warp == kKMmaWarp) {
    tmem_alloc(tmem_slot, 128 * kKNumD);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto job_rank = [&](int j, int& kv) -> int {
    kv = (grp * G + j % G) / qpk;
    return lay.k_rank[kv];
  };
  long long* trace = (p.trace && split == 0 && grp == 0 && b < 2) ? p.trace + (int64_t)b * p.trace_jobs * kTrFields
                                                                  : nullptr;
  auto stamp = [&](int j, int f) {
    if (trace && j < p.trace_jobs) trace[(int64_t)j * kTrFields + f] = clock64();
  };
  auto fail = [&](int code) {
    record_error(p.err, code);
    *s_abort = 1;
  };
  // Converter threads: issue this thread's row of job j's codes as 16-byte
  // copies (one commit group per job, empty past the last job).
  auto issue_copies = [&](int j) {
    if (j < J) {
      int kv;
      const int r = job_rank(j, kv);
      const int t0 = t_begin + (j / G) * 128;
      if (t0 + tid < t_end) {
        const int rc = (r * XB) >> 4;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.k_cache) +
                             (lay.k_offset[kv] + (int64_t)b * lay.k_batch_stride[kv] + (int64_t)(t0 + tid) * r) * XB;
        uint8_t* dst = Ssm + (size_t)(j % STG) * slot_bytes + (size_t)tid * k_pitch16(r, XB) * 16;
#pragma unroll 4
        for (int c = 0; c < rc; ++c) cp_async16(dst + c * 16, src + c * 16);
      }
    }
    cp_async_commit();
  };

  if (warp < kKConvWarps)
    for (int j = 0; j < STG - 1; ++j) issue_copies(j);

  if (warp < kKConvWarps + kKDrainWarps) {
    // ---- build W_g = [P | Q] (fp16, canonical K-major layout) for each head of
    // the group while the first codes stream in.
    const int wt = tid;  // 0..255
    for (int e = wt; e < G * 128; e += kKWorkers)
      s_q[e] = load_as_f32(p.q, p.q_dtype, ((int64_t)b * Hq + grp * G) * 128 + e);
    if (wt < 64) {
      float c, sn;
      exact_sincos(128, p.inv_freq[wt], c, sn);
      s_rot[wt] = make_float2(c, sn);
    }
    named_bar_sync(2, kKWorkers);
    for (int g = 0; g < G; ++g) {
      const int qh = grp * G + g, kv = qh / qpk, r = lay.k_rank[kv];
      const float* qv = s_q + g * 128;
      float* scr = reinterpret_cast<float*>(Asm);  // [128][r] fp32 scratch (fits the A buffers)
      const int64_t ubase = (int64_t)128 * lay.k_col[kv];
      float amax = 0.f;
      for (int e = wt; e < r * 64; e += kKWorkers) {
        const int i = e / r, c = e - i * r;          // c fastest: coalesced U rows
        const float u1 = load_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)i * r + c);
        const float u2 = load_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)(i + 64) * r + c);
        const float sc = QUANT ? __half2float(p.k_scales[(int64_t)b * lay.k_rank_total + lay.k_col[kv] + c]) : 1.f;
        const float qa = qv[i], qb = qv[i + 64];
        const float P = sc * (qa * u1 + qb * u2);
        const float Q = sc * (qb * u1 - qa * u2);
        scr[i * r + c] = P;
        scr[(64 + i) * r + c] = Q;
        amax = fmaxf(amax, fmaxf(fabsf(P), fabsf(Q)));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0) s_red[warp] = amax;
      named_bar_sync(2, kKWorkers);
      amax = 0.f;
      for (int w = 0; w < kKConvWarps + kKDrainWarps; ++w) amax = fmaxf(amax, s_red[w]);
      // Power-of-two normalisation: the largest entries of W land in [2^13, 2^14],
      // keeping fp16's full precision; undone exactly in the drain.
      const float eta = amax > 0.f ? exp2f(ceilf(log2f(amax)) - 14.f) : 1.f;
      const float inv_eta = 1.f / eta;
      if (wt == 0) s_epi[g] = eta * p.out_scale;
      uint8_t* Bg = Bsm + s_boff[g];
      const int nc = r >> 3;
      for (int e = wt; e < 128 * nc; e += kKWorkers) {
        const int n = e & 127, kc = e >> 7;
        const float4 f0 = *reinterpret_cast<const float4*>(scr + n * r + kc * 8);
        const float4 f1 = *reinterpret_cast<const float4*>(scr + n * r + kc * 8 + 4);
        __half2 h0 = __floats2half2_rn(f0.x * inv_eta, f0.y * inv_eta), h1 = __floats2half2_rn(f0.z * inv_eta, f0.w * inv_eta);
        __half2 h2 = __floats2half2_rn(f1.x * inv_eta, f1.y * inv_eta), h3 = __floats2half2_rn(f1.z * inv_eta, f1.w * inv_eta);
        *reinterpret_cast<uint4*>(Bg + (n >> 3) * (r * 16) + kc * 128 + (n & 7) * 16) =
            make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                       *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
      }
      fence_proxy_async_smem();
      named_bar_sync(2, kKWorkers);                  // scratch reuse + s_red reuse
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(w_ready);
  }

  if (warp == kKMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_f16_f32(128, 128);
      if (!mbar_wait(w_ready, 0)) fail(kDevWaitMma);
      for (int j = 0; j < J && !*s_abort; ++j) {
        const int ka = j % kKNumA, kd = j % kKNumD;
        if (!mbar_wait(a_full + ka, (uint32_t)((j / kKNumA) & 1))) { fail(kDevWaitMma); break; }
        if (!mbar_wait(d_empty + kd, (uint32_t)(((j / kKNumD) & 1) ^ 1))) { fail(kDevWaitMma); break; }
        tc_fence_after();
        stamp(j, kTrMmaIssue);
        int kv;
        const int r = job_rank(j, kv);
        const uint32_t a0 = smem_u32(Asm + (size_t)ka * rmax * 256);
        const uint32_t b0 = smem_u32(Bsm + s_boff[j % G]);
        const uint32_t sbo = (uint32_t)r * 16u;
        const uint32_t d = tmem + (uint32_t)kd * 128u;
        for (int k = 0; k < r / 16; ++k)
          mma_f16_ss(d, smem_desc(a0 + k * 256, 128, sbo), smem_desc(b0 + k * 256, 128, sbo), IDESC, k > 0 ? 1u : 0u);
        mma_commit(a_empty + ka);
        mma_commit(d_full + kd);
      }
    }
  } else if (warp < kKConvWarps) {
    // ------------------------------------------------------------ converters
    const int row = tid;  // one token row per converter thread
    for (int j = 0; j < J; ++j) {
      const int ka = j % kKNumA;
      if (tid == 0) stamp(j, kTrConvBegin);
      cp_async_wait<STG - 2>();                       // this thread's copies of job j landed
      named_bar_sync(3, 32 * kKConvWarps);            // ... and every other converter's
      if (tid == 0) stamp(j, kTrConvLanded);
      if (*s_abort) break;
      issue_copies(j + STG - 1);                      // refill the slot read in iteration j-1
      if (!mbar_wait(a_empty + ka, (uint32_t)(((j / kKNumA) & 1) ^ 1))) { fail(kDevWaitMma); break; }
      if (tid == 0) stamp(j, kTrConvAEmpty);
      int kv;
      const int r = job_rank(j, kv);
      const int t0 = t_begin + (j / G) * 128;
      const int n = min(128, t_end - t0);
      const int rc = (r * XB) >> 4;
      const uint8_t* srow = Ssm + (size_t)(j % STG) * slot_bytes + (size_t)row * k_pitch16(r, XB) * 16;
      uint8_t* arow = Asm + (size_t)ka * rmax * 256 + (row >> 3) * (r * 16) + (row & 7) * 16;
      constexpr int KPC = kc_per_chunk<XT>();
      constexpr int MAXC = (STARKV_MAX_K_RANK * XB) / 16;
      uint4 w[MAXC];
#pragma unroll
      for (int c = 0; c < MAXC; ++c)
        if (c < rc) w[c] = row < n ? *reinterpret_cast<const uint4*>(srow + c * 16) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int c = 0; c < MAXC; ++c)
        if (c < rc) cvt_chunk<XT>(w[c], arow, c * KPC);
      if (tid == 0) stamp(j, kTrConvCvt);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full + ka);
      if (tid == 0) stamp(j, kTrConvDone);
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------------ drain
    const int dw = warp - kKConvWarps;       // 0..3 == TMEM lane quarter (warp % 4)
    const int row = dw * 32 + lane;
    float m_run[4] = {kNegBig, kNegBig, kNegBig, kNegBig};
    float l_run[4] = {0.f, 0.f, 0.f, 0.f};
    float cs_c[64], cs_s[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) exact_sincos(t_begin + row, p.inv_freq[i], cs_c[i], cs_s[i]);
    for (int j = 0; j < J; ++j) {
      if (*s_abort) break;
      const int tile = j / G, g = j % G, kd = j % kKNumD;
      const int l = t_begin + tile * 128 + row;
      const bool valid = l < t_end;
      if (g == 0 && tile > 0) {
        // advance every frequency by 128 positions
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float2 rt = s_rot[i];
          const float c = cs_c[i], sn = cs_s[i];
          cs_c[i] = fmaf(c, rt.x, -sn * rt.y);
          cs_s[i] = fmaf(sn, rt.x, c * rt.y);
        }
      }
      if (row == 0) stamp(j, kTrDrainWait);
      if (!mbar_wait(d_full + kd, (uint32_t)((j / kKNumD) & 1))) { fail(kDevWaitMma); break; }
      tc_fence_after();
      if (row == 0) stamp(j, kTrDrainGot);
      const uint32_t taddr = tmem + ((uint32_t)(dw * 32) << 16) + (uint32_t)kd * 128u;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float va[32], vc[32];
        tmem_ld16x4(taddr + 32 * k, taddr + 32 * k + 16, taddr + 64 + 32 * k, taddr + 80 + 32 * k, va, va + 16, vc,
                    vc + 16);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          a0 = fmaf(cs_c[32 * k + i], va[i], a0);
          a1 = fmaf(cs_c[32 * k + i + 1], va[i + 1], a1);
          a2 = fmaf(cs_s[32 * k + i], vc[i], a2);
          a3 = fmaf(cs_s[32 * k + i + 1], vc[i + 1], a3);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_empty + kd);
      if (valid) {
        const int qh = grp * G + g;
        float val = ((a0 + a1) + (a2 + a3)) * s_epi[g];
        if (p.mask) val = fmaf(p.mask[(int64_t)b * p.T + l], p.mask_scale, val);
        p.logits[((int64_t)b * Hq + qh) * p.T + l] = val;
#pragma unroll
        for (int gg = 0; gg < 4; ++gg)
          if (gg == g) softmax_merge(m_run[gg], l_run[gg], val, 1.f);
      }
      if (row == 0) stamp(j, kTrDrainDone);
    }
    // split statistics: (max, sum exp2(logit - max)) per head over this split
    if (p.stats) {
      float* s_m = s_red;          // [4 heads][4 warps]
      float* s_l = s_red + 16;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float m = m_run[g], lsum = l_run[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, lsum, o);
          softmax_merge(m, lsum, m2, l2);
        }
        if (lane == 0) { s_m[g * 4 + dw] = m; s_l[g * 4 + dw] = lsum; }
      }
      named_bar_sync(1, 32 * kKDrainWarps);
      if (dw == 0 && lane < G && !*s_abort) {
        float M = s_m[lane * 4], Lsum = s_l[lane * 4];
        for (int w = 1; w < 4; ++w) softmax_merge(M, Lsum, s_m[lane * 4 + w], s_l[lane * 4 + w]);
        p.stats[((int64_t)b * Hq + grp * G + lane) * p.nsplit + split] = make_float2(M, Lsum);
      }
    }
  }

  // ---- teardown: no MMA of ours may still be writing TMEM when it is released.
  tc_fence_before();
  __syncthreads();
  if (warp == kKMmaWarp) {
    if (lane == 0) {
      mma_commit(fin_bar);                    // arrives once all MMAs issued so far have retired
      (void)mbar_wait(fin_bar, 0);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128 * kKNumD);
  }
}

}  // namespace starkv
