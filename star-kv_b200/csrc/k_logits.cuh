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
// CTA = (sequence split, group of G query heads, sequence b), 512 threads.  A
// "job" is one (128-token tile, head) pair.  Two pipelines work on alternate
// tiles; each is a converter warpgroup and a drain warpgroup handing off through
// mbarriers, so copy, conversion, MMA and drain of different jobs overlap:
//   converter warpgroup: the leader bulk-prefetches jobs several steps ahead
//                    into L2; every thread cp.async's its token row of the next
//                    job into a staging slot (rows padded to an odd number of
//                    16-byte chunks: conflict-free row reads), converts the
//                    current job's codes to fp16 in the canonical no-swizzle
//                    K-major A layout, and the leader issues r/16 tcgen05.mma
//                    (M=128, N=128, K=16) into the pipeline's TMEM accumulator;
//   drain warpgroup: tcgen05.ld of the accumulator row of its token, the
//                    RoPE-weighted reduction, mask, logits to global, and an
//                    online (max, sum exp2) per head for the split-softmax merge.
// setmaxnreg moves registers from the converters (80) to the drains (176).
//
// RoPE angles: each drain thread owns one token row of its pipeline's tiles; it
// starts from cos/sin of l*w_i for its first token and advances by the exact
// rotation through 256*w_i per tile (fp32, 4 FMA per frequency per tile,
// shared by the G heads).  The angles are the exact l*w_i; the reference's fp32 product
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
  int pitch16max;         // largest staging row pitch (16-byte units) over the heads
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

// Two pipelines per CTA work on alternate 128-token tiles: warpgroups 0/1
// convert (and their leader thread issues the MMAs), warpgroups 2/3 drain.
constexpr int kKPipes = 2;
constexpr int kKThreads = 512;
constexpr int kKConvRegs = 80, kKDrainRegs = 176;   // 256*80 + 256*176 = 512 * 128 (launch budget)
constexpr int kKStages = 2;      // staging slots per pipeline for 1-/2-byte latents (deeper prefetch goes to L2)
constexpr int kKPrefetch = 6;    // pipeline jobs ahead that are prefetched into L2
constexpr int kKHeader = 2048;   // barriers / scratch at the start of dynamic smem

// fp32 latents (4x the bytes of int8 codes) use one staging slot per pipeline.
__host__ __device__ constexpr int k_stages(int xbytes) { return xbytes == 4 ? 1 : kKStages; }

// Staging row pitch in 16-byte units.  Rows whose chunk count is a multiple of 4
// would put 4+ rows of a quarter-warp on the same banks: they get one chunk of
// padding; other counts conflict at most 2-way and stay unpadded.
__host__ __device__ inline int k_pitch16(int r, int xbytes) {
  const int rc = (r * xbytes) >> 4;
  return (rc & 3) == 0 ? rc + 1 : rc;
}

__host__ __device__ inline size_t k_smem_bytes(int bsum, int rmax, int pitch16max, int xbytes) {
  return (size_t)kKHeader + (size_t)bsum * 256 + (size_t)kKPipes * 2 * rmax * 256 +
         (size_t)kKPipes * k_stages(xbytes) * 128 * pitch16max * 16;
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

// Convert one staged row of RC 16-byte chunks into the A row (compile-time trip count).
template <typename XT, int RC>
__device__ __forceinline__ void convert_row(const uint8_t* srow, uint8_t* arow, bool valid) {
  uint4 w[RC];
#pragma unroll
  for (int c = 0; c < RC; ++c) w[c] = valid ? *reinterpret_cast<const uint4*>(srow + c * 16) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int c = 0; c < RC; ++c) cvt_chunk<XT>(w[c], arow, c * kc_per_chunk<XT>());
}

// A-row byte offset of staging chunk c (each staging chunk is 16 bytes of latents).
template <typename XT>
__device__ __forceinline__ int a_offset_of_chunk(int c) { return (c * (16 / (int)sizeof(XT))) / 8 * 128; }

template <typename XT>
__device__ __forceinline__ void convert_tail(int n, const uint8_t* srow, uint8_t* arow, bool valid) {
  switch (n) {
    case 1: convert_row<XT, 1>(srow, arow, valid); break;
    case 2: convert_row<XT, 2>(srow, arow, valid); break;
    case 3: convert_row<XT, 3>(srow, arow, valid); break;
    case 4: convert_row<XT, 4>(srow, arow, valid); break;
    case 5: convert_row<XT, 5>(srow, arow, valid); break;
    case 6: convert_row<XT, 6>(srow, arow, valid); break;
    case 7: convert_row<XT, 7>(srow, arow, valid); break;
    default: break;
  }
}

// Convert a staged row of rc chunks: whole groups of 8 chunks, then the remainder
// (fp32 chunks hold half an A chunk; 8 of them always end on an A-chunk boundary).
template <typename XT>
__device__ __forceinline__ void convert_row_rc(int rc, const uint8_t* srow, uint8_t* arow, bool valid) {
  int c = 0;
  for (; c + 8 <= rc; c += 8) convert_row<XT, 8>(srow + c * 16, arow + a_offset_of_chunk<XT>(c), valid);
  if (c < rc) convert_tail<XT>(rc - c, srow + c * 16, arow + a_offset_of_chunk<XT>(c), valid);
}

template <typename XT, bool QUANT, int G>
__global__ void __launch_bounds__(kKThreads, 1) k_logits_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wg = warp >> 2;                      // warpgroup 0..3
  const int split = blockIdx.x, grp = blockIdx.y, b = blockIdx.z;
  const starkv_layout& lay = p.lay;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int rmax = p.rmax;
  const int t_begin = split * p.tps;
  const int t_end = min(p.T, t_begin + p.tps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + 127) / 128 : 0;
  constexpr int XB = (int)sizeof(XT);
  constexpr int STG = k_stages(XB);

  // ---- shared memory carve-up (barriers per pipeline: a_full[2] a_empty[2] d_full[2] d_empty[2])
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* fin_bar = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 256);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 260);
  int* s_boff = reinterpret_cast<int*>(smem + 272);           // [4] byte offset of W_g
  int* s_rank = reinterpret_cast<int*>(smem + 288);           // [4] rank of head g
  const uint8_t** s_src = reinterpret_cast<const uint8_t**>(smem + 320);  // [4] codes of (b, kv(g)) at slot 0
  float* s_epi = reinterpret_cast<float*>(smem + 352);        // [4]
  float* s_red = reinterpret_cast<float*>(smem + 384);        // [64]
  float2* s_rot = reinterpret_cast<float2*>(smem + 640);      // [64] rotation by 256 positions
  uint8_t* Bsm = smem + kKHeader;
  uint8_t* Asm = Bsm + (size_t)p.bsum * 256;                                // [pipe][2]
  uint8_t* Ssm = Asm + (size_t)kKPipes * 2 * rmax * 256;                    // [pipe][stage]
  const uint32_t abuf_bytes = (uint32_t)rmax * 256u;
  const uint32_t slot_bytes = 128u * p.pitch16max * 16u;

  if (tid == 0) {
    for (int pp = 0; pp < kKPipes; ++pp) {
      uint64_t* pb = bars + 8 * pp;
      for (int k = 0; k < 2; ++k) {
        mbar_init(pb + k, 4);          // a_full: 4 converter warps
        mbar_init(pb + 2 + k, 1);      // a_empty: MMA commit
        mbar_init(pb + 4 + k, 1);      // d_full: MMA commit
        mbar_init(pb + 6 + k, 4);      // d_empty: 4 drain warps
      }
    }
    mbar_init(fin_bar, kKPipes);
    *s_abort = 0;
    int off = 0;
    for (int g = 0; g < G; ++g) {
      const int kv = (grp * G + g) / qpk;
      s_boff[g] = off;
      s_rank[g] = lay.k_rank[kv];
      s_src[g] = reinterpret_cast<const uint8_t*>(p.k_cache) + (lay.k_offset[kv] + (int64_t)b * lay.k_batch_stride[kv]) * XB;
      off += lay.k_rank[kv] * 256;
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  long long* trace = (p.trace && split == 0 && grp == 0 && b < 2) ? p.trace + (int64_t)b * p.trace_jobs * kTrFields
                                                                  : nullptr;
  auto stamp = [&](int j, int f) {
    if (trace && j < p.trace_jobs) trace[(int64_t)j * kTrFields + f] = clock64();
  };
  auto fail = [&](int code) {
    record_error(p.err, code);
    *s_abort = 1;
  };

  // ---- build W_g = [P | Q] (fp16, canonical K-major layout) for each head (all threads)
  {
    float* s_qall = reinterpret_cast<float*>(Ssm);            // [G][128] in the staging area (free now)
    for (int e = tid; e < G * 128; e += kKThreads)
      s_qall[e] = load_as_f32(p.q, p.q_dtype, ((int64_t)b * Hq + grp * G) * 128 + e);
    if (tid < 64) {
      float c, sn;
      exact_sincos(128 * kKPipes, p.inv_freq[tid], c, sn);
      s_rot[tid] = make_float2(c, sn);
    }
    __syncthreads();
    for (int g = 0; g < G; ++g) {
      const int qh = grp * G + g, kv = qh / qpk, r = lay.k_rank[kv];
      const float* qv = s_qall + g * 128;
      float* scr = reinterpret_cast<float*>(Asm);  // [128][r] fp32 scratch (fits the A buffers)
      const int64_t ubase = (int64_t)128 * lay.k_col[kv];
      float amax = 0.f;
      for (int e = tid; e < r * 64; e += kKThreads) {
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
      __syncthreads();
      amax = 0.f;
      for (int w = 0; w < kKThreads / 32; ++w) amax = fmaxf(amax, s_red[w]);
      // Power-of-two normalisation: the largest entries of W land in [2^13, 2^14],
      // keeping fp16's full precision; undone exactly in the drain.
      const float eta = amax > 0.f ? exp2f(ceilf(log2f(amax)) - 14.f) : 1.f;
      const float inv_eta = 1.f / eta;
      if (tid == 0) s_epi[g] = eta * p.out_scale;
      uint8_t* Bg = Bsm + s_boff[g];
      const int nc = r >> 3;
      for (int e = tid; e < 128 * nc; e += kKThreads) {
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
      __syncthreads();                             // scratch reuse + s_red reuse
    }
  }

  if (wg < kKPipes) {
    // ============================================================ converter pipeline `pipe`
    regs_dec<kKConvRegs>();
    const int pipe = wg;
    const int ct = tid & 127;                      // token row of this thread
    uint64_t* pb = bars + 8 * pipe;
    const int my_tiles = ntiles > pipe ? (ntiles - pipe + kKPipes - 1) / kKPipes : 0;
    const int K = my_tiles * G;                    // jobs of this pipeline
    auto job_tile = [&](int k) { return pipe + kKPipes * (k / G); };
    auto issue_copies = [&](int k) {
      if (k < K) {
        const int g = k % G, r = s_rank[g];
        const int t0 = t_begin + job_tile(k) * 128;
        if (t0 + ct < t_end) {
          const int rc = (r * XB) >> 4;
          const uint8_t* src = s_src[g] + (size_t)(t0 + ct) * r * XB;
          uint8_t* dst = Ssm + (size_t)(pipe * STG + (k % STG)) * slot_bytes + (size_t)ct * k_pitch16(r, XB) * 16;
#pragma unroll 4
          for (int c = 0; c < rc; ++c) cp_async16(dst + c * 16, src + c * 16);
        }
      }
      cp_async_commit();
    };
    auto prefetch = [&](int k) {
      if (k < K) {
        const int g = k % G, r = s_rank[g];
        const int t0 = t_begin + job_tile(k) * 128;
        const int n = min(128, t_end - t0);
        bulk_prefetch_l2(s_src[g] + (size_t)t0 * r * XB, (uint32_t)(n * r * XB));
      }
    };
    const bool leader = ct == 0;
    if (leader)
      for (int k = 0; k < kKPrefetch; ++k) prefetch(k);
    issue_copies(0);
    constexpr uint32_t IDESC = idesc_f16_f32(128, 128);
    for (int k = 0; k < K; ++k) {
      const int kb = k & 1;
      const int j = job_tile(k) * G + (k % G);     // global job index (trace)
      if (leader) stamp(j, kTrConvBegin);
      cp_async_wait<0>();                          // this thread's copies of job k landed
      named_bar_sync(3 + pipe, 128);               // ... and every other converter's of this pipeline
      if (leader) stamp(j, kTrConvLanded);
      if (*s_abort) break;
      if (STG > 1) issue_copies(k + 1);            // refill the slot read in iteration k-1
      if (leader) prefetch(k + kKPrefetch);
      if (!mbar_wait(pb + 2 + kb, (uint32_t)(((k >> 1) & 1) ^ 1))) { fail(kDevWaitMma); break; }
      if (leader) stamp(j, kTrConvAEmpty);
      const int g = k % G, r = s_rank[g];
      const int t0 = t_begin + job_tile(k) * 128;
      const int rc = (r * XB) >> 4;
      const uint8_t* srow = Ssm + (size_t)(pipe * STG + (k % STG)) * slot_bytes + (size_t)ct * k_pitch16(r, XB) * 16;
      uint8_t* A = Asm + (size_t)(pipe * 2 + kb) * abuf_bytes;
      uint8_t* arow = A + (ct >> 3) * (r * 16) + (ct & 7) * 16;
      convert_row_rc<XT>(rc, srow, arow, t0 + ct < t_end);
      if (leader) stamp(j, kTrConvCvt);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(pb + kb);
      if (STG == 1) {                              // single slot: refill once every row was read
        named_bar_sync(3 + pipe, 128);
        issue_copies(k + 1);
      }
      if (leader) {
        stamp(j, kTrConvDone);
        // ---- issue the MMA of job k once all 4 warps wrote A and the drain freed the accumulator
        if (!mbar_wait(pb + kb, (uint32_t)((k >> 1) & 1))) { fail(kDevWaitMma); break; }
        if (!mbar_wait(pb + 6 + kb, (uint32_t)(((k >> 1) & 1) ^ 1))) { fail(kDevWaitMma); break; }
        tc_fence_after();
        stamp(j, kTrMmaIssue);
        const uint32_t a0 = smem_u32(A);
        const uint32_t b0 = smem_u32(Bsm + s_boff[g]);
        const uint32_t sbo = (uint32_t)r * 16u;
        const uint32_t d = tmem + (uint32_t)(pipe * 2 + kb) * 128u;
        for (int kk = 0; kk < r / 16; ++kk)
          mma_f16_ss(d, smem_desc(a0 + kk * 256, 128, sbo), smem_desc(b0 + kk * 256, 128, sbo), IDESC, kk > 0 ? 1u : 0u);
        mma_commit(pb + 2 + kb);
        mma_commit(pb + 4 + kb);
      }
    }
    cp_async_wait<0>();
    if (leader) {
      mma_commit(fin_bar);                         // arrives once this thread's MMAs retired
      if (!mbar_wait(fin_bar, 0)) fail(kDevWaitMma);
    }
  } else {
    // ============================================================ drain pipeline `pipe`
    regs_inc<kKDrainRegs>();
    const int pipe = wg - kKPipes;
    const int dw = warp & 3;                       // TMEM lane quarter (warp % 4)
    const int row = dw * 32 + lane;
    uint64_t* pb = bars + 8 * pipe;
    const int my_tiles = ntiles > pipe ? (ntiles - pipe + kKPipes - 1) / kKPipes : 0;
    const int K = my_tiles * G;
    float m_run[G], l_run[G];
#pragma unroll
    for (int g = 0; g < G; ++g) { m_run[g] = kNegBig; l_run[g] = 0.f; }
    float cs_c[64], cs_s[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) exact_sincos(t_begin + pipe * 128 + row, p.inv_freq[i], cs_c[i], cs_s[i]);
    for (int k = 0; k < K; ++k) {
      if (*s_abort) break;
      const int kb = k & 1, g = k % G;
      const int tile = pipe + kKPipes * (k / G);
      const int j = tile * G + g;
      const int l = t_begin + tile * 128 + row;
      if (g == 0 && k > 0) {
        // advance every frequency by 256 positions (this pipeline's tile stride)
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float2 rt = s_rot[i];
          const float c = cs_c[i], sn = cs_s[i];
          cs_c[i] = fmaf(c, rt.x, -sn * rt.y);
          cs_s[i] = fmaf(sn, rt.x, c * rt.y);
        }
      }
      if (row == 0) stamp(j, kTrDrainWait);
      if (!mbar_wait(pb + 4 + kb, (uint32_t)((k >> 1) & 1))) { fail(kDevWaitMma); break; }
      tc_fence_after();
      if (row == 0) stamp(j, kTrDrainGot);
      const uint32_t taddr = tmem + ((uint32_t)(dw * 32) << 16) + (uint32_t)(pipe * 2 + kb) * 128u;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float va[16], vc[16];
        tmem_ld16x2(taddr + 16 * q, taddr + 64 + 16 * q, va, vc);
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          a0 = fmaf(cs_c[16 * q + i], va[i], a0);
          a1 = fmaf(cs_c[16 * q + i + 1], va[i + 1], a1);
          a2 = fmaf(cs_s[16 * q + i], vc[i], a2);
          a3 = fmaf(cs_s[16 * q + i + 1], vc[i + 1], a3);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pb + 6 + kb);
      if (l < t_end) {
        const int qh = grp * G + g;
        float val = ((a0 + a1) + (a2 + a3)) * s_epi[g];
        if (p.mask) val = fmaf(p.mask[(int64_t)b * p.T + l], p.mask_scale, val);
        p.logits[((int64_t)b * Hq + qh) * p.T + l] = val;
#pragma unroll
        for (int gg = 0; gg < G; ++gg)
          if (gg == g) softmax_merge(m_run[gg], l_run[gg], val, 1.f);
      }
      if (row == 0) stamp(j, kTrDrainDone);
    }
    // warp-level (max, sum exp2) per head -> s_red[g][drain warp]
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float m = m_run[g], lsum = l_run[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, lsum, o);
        softmax_merge(m, lsum, m2, l2);
      }
      if (lane == 0) { s_red[g * 8 + pipe * 4 + dw] = m; s_red[32 + g * 8 + pipe * 4 + dw] = lsum; }
    }
  }

  // ---- split statistics and teardown (every MMA has retired: both issuers waited fin_bar)
  tc_fence_before();
  __syncthreads();
  if (p.stats && tid < G && !*s_abort) {
    float M = s_red[tid * 8], Lsum = s_red[32 + tid * 8];
    for (int w = 1; w < 8; ++w) softmax_merge(M, Lsum, s_red[tid * 8 + w], s_red[32 + tid * 8 + w]);
    p.stats[((int64_t)b * Hq + grp * G + tid) * p.nsplit + split] = make_float2(M, Lsum);
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace starkv
