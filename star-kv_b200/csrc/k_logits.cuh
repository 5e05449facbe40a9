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
// CTA = (sequence split, group of G query heads, sequence b), 512 threads, one
// CTA per SM (it owns the 512 TMEM columns).  A "unit" is one 128-token tile of
// one KV head (the G heads form runs of heads that share a KV head); a "job" is
// one (tile, query head) pair.  Roles, handing off through mbarriers:
//   producer warp:   coalesced 16-byte cp.async of a unit's latent rows (one
//                    contiguous block in HBM) into a ring of shared-memory stages,
//                    rows padded to an odd number of 16-byte chunks so that
//                    row-per-thread reads are conflict-free; each lane's copies
//                    arrive on the stage's mbarrier when they complete;
//   converter warpgroup: thread = token row; reads its staged row, converts to
//                    fp16 (int8 codes are exact in fp16) and writes it into one
//                    of 4 A buffers in TMEM with tcgen05.st — the A operand never
//                    touches shared memory;
//   MMA thread:      per job r/16 tcgen05.mma (A from TMEM, B = W_g from shared
//                    memory, M=128, N=128, K=16) into one of 2 TMEM accumulators;
//   drain warpgroups: both take every job; warpgroup h owns the frequencies
//                    [32h, 32h + 32): one tcgen05.ld of its token's 64 accumulator
//                    columns (the accumulator is released right after) and the
//                    RoPE-weighted partial sum (packed fp32x2 FMA) into a ring of
//                    partials in shared memory;
//   finaliser warps 2, 3 (alternate jobs): sum of the two partials, scale, mask,
//                    logits to global, and a running maximum per head — the split
//                    maximum the V kernel's softmax starts from (the V kernel forms
//                    the exponentials and their sums itself).
// TMEM columns: [0, 256) the two accumulators, [256, 512) four A buffers of 64
// columns (r <= 128 fp16 values per row).
//
// RoPE angles: each drain thread owns one token row; it starts from cos/sin of
// l*w_i for its first token and advances by the exact rotation through
// 128*w_i when its tile changes (fp32, 4 FMA per frequency per tile,
// shared by the heads of the tile).  The angles are the exact l*w_i; the
// reference's fp32 product fl(l*w_i) differs from them by at most half an ulp of
// the angle.
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
  float* smax;            // (B, Hq, nsplit) maximum logit of each split, or null
  int* err;
  int q_dtype, w_dtype;
  int T, nsplit, tps;     // tokens, splits, tokens per split (multiple of 128)
  int G, rmax, bsum;      // heads per CTA, max rank, max per-group rank sum (W matrices in smem)
  int pitch16max;         // largest staging row pitch (16-byte units) over the heads
  int nstages;            // staging ring depth
  float out_scale;        // multiplier of q.k (scaling * log2 e for decode)
  float mask_scale;       // multiplier of the mask (log2 e for decode)
  const uint8_t* wpre;    // W of every (sequence, query head) from k_wprep_kernel (stride wstride), or null:
  const float* weta;      //   then the CTA builds its W itself; eta of every (sequence, query head)
  int wstride;            // bytes per (sequence, query head) W image
  long long* trace;       // optional per-job clock64 timeline of CTAs (0, 0, b < 2); null = off
  int trace_jobs;         // jobs recorded per traced CTA
};

// Per-job timeline fields (clock64 of the SM).
enum KTrace {
  kTrLoadIssue = 0, kTrConvBegin, kTrConvAEmpty, kTrConvDone, kTrMmaIssue, kTrDrainWait, kTrDrainGot,
  kTrDrainDone, kTrDrainLd, kTrFields = 10
};

constexpr int kKThreads = 512;
// Register budget per warpgroup after setmaxnreg: producer/MMA, converter, 2 drains.
constexpr int kKCtlRegs = 56, kKConvRegs = 120, kKDrainRegs = 168;  // 56 + 120 + 2*168 = 4 * 128 (launch budget)
constexpr int kKMaxStages = 8;   // staging ring depth (bounded by shared memory)
constexpr int kKAbufs = 4;       // A buffers in TMEM
constexpr int kKAcc = 2;         // accumulators in TMEM
constexpr int kKPartRing = 8;    // partial-logit slots between the two drain warpgroups
constexpr int kKHeader = 12288;  // barriers / scratch / partial-logit ring at the start of dynamic smem
constexpr int kKSmemMax = 227 * 1024;

// Staging row pitch in 16-byte units.  Rows whose chunk count is a multiple of 4
// would put 4+ rows of a quarter-warp on the same banks: they get one chunk of
// padding; other counts conflict at most 2-way and stay unpadded.
__host__ __device__ inline int k_pitch16(int r, int xbytes) {
  const int rc = (r * xbytes) >> 4;
  return (rc & 3) == 0 ? rc + 1 : rc;
}

__host__ __device__ inline size_t k_stage_bytes(int pitch16max) { return (size_t)128 * pitch16max * 16; }

__host__ __device__ inline size_t k_smem_bytes(int bsum, int pitch16max, int nstages) {
  return (size_t)kKHeader + (size_t)bsum * 256 + (size_t)nstages * k_stage_bytes(pitch16max);
}

// Staging depth that fits next to the W matrices (0 when fewer than 2 fit).
__host__ __device__ inline int k_stages_fit(int bsum, int pitch16max) {
  const long avail = (long)kKSmemMax - kKHeader - (long)bsum * 256;
  long ns = avail > 0 ? avail / (long)k_stage_bytes(pitch16max) : 0;
  if (ns > kKMaxStages) ns = kKMaxStages;
  return ns >= 2 ? (int)ns : 0;
}

// 8 int8 codes -> 8 fp16 (exact): x -> (x + 128) as a byte; 0x64XX as fp16 is
// 1024 + XX; subtract 1152.
__device__ __forceinline__ void cvt8_i8(uint32_t lo, uint32_t hi, uint32_t* o) {
  const uint32_t a = lo ^ 0x80808080u, b = hi ^ 0x80808080u;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
  uint32_t t;
  __half2 h;
  t = __byte_perm(a, 0x64646464u, 0x5140); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o[0] = *reinterpret_cast<uint32_t*>(&h);
  t = __byte_perm(a, 0x64646464u, 0x7362); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o[1] = *reinterpret_cast<uint32_t*>(&h);
  t = __byte_perm(b, 0x64646464u, 0x5140); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o[2] = *reinterpret_cast<uint32_t*>(&h);
  t = __byte_perm(b, 0x64646464u, 0x7362); h = __hsub2(*reinterpret_cast<__half2*>(&t), bias); o[3] = *reinterpret_cast<uint32_t*>(&h);
}

// TMEM columns (packed fp16 pairs) produced by one 16-byte staging chunk.
template <typename XT>
__host__ __device__ constexpr int k_cols_per_chunk() { return 8 / (int)sizeof(XT); }

// Convert one 16-byte staging chunk to packed fp16 pairs and store them at
// TMEM address `taddr` (this warp's lanes, consecutive columns).
template <typename XT>
__device__ __forceinline__ void cvt_store(const uint4 w, uint32_t taddr);

template <>
__device__ __forceinline__ void cvt_store<int8_t>(const uint4 w, uint32_t taddr) {
  uint32_t o[8];
  cvt8_i8(w.x, w.y, o);
  cvt8_i8(w.z, w.w, o + 4);
  tmem_st8(taddr, o);
}
template <>
__device__ __forceinline__ void cvt_store<__half>(const uint4 w, uint32_t taddr) {
  const uint32_t o[4] = {w.x, w.y, w.z, w.w};
  tmem_st4(taddr, o);
}
template <>
__device__ __forceinline__ void cvt_store<__nv_bfloat16>(const uint4 w, uint32_t taddr) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float lo = __uint_as_float(in[k] << 16), hi = __uint_as_float(in[k] & 0xFFFF0000u);
    __half2 h = __floats2half2_rn(lo, hi);
    o[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  tmem_st4(taddr, o);
}
template <>
__device__ __forceinline__ void cvt_store<float>(const uint4 w, uint32_t taddr) {
  __half2 h0 = __floats2half2_rn(__uint_as_float(w.x), __uint_as_float(w.y));
  __half2 h1 = __floats2half2_rn(__uint_as_float(w.z), __uint_as_float(w.w));
  const uint32_t o[2] = {*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1)};
  tmem_st2(taddr, o);
}

// Convert N staged chunks (loads first, then conversions and stores).
template <typename XT, int N>
__device__ __forceinline__ void convert_chunks(const uint8_t* srow, uint32_t taddr) {
  uint4 w[N];
#pragma unroll
  for (int c = 0; c < N; ++c) w[c] = *reinterpret_cast<const uint4*>(srow + c * 16);
#pragma unroll
  for (int c = 0; c < N; ++c) cvt_store<XT>(w[c], taddr + c * k_cols_per_chunk<XT>());
}

// Convert a staged row of rc chunks into TMEM: groups of 8 chunks, then the rest.
template <typename XT>
__device__ __forceinline__ void convert_row(int rc, const uint8_t* srow, uint32_t taddr) {
  int c = 0;
  for (; c + 8 <= rc; c += 8) convert_chunks<XT, 8>(srow + c * 16, taddr + c * k_cols_per_chunk<XT>());
  const uint8_t* s = srow + c * 16;
  const uint32_t t = taddr + c * k_cols_per_chunk<XT>();
  switch (rc - c) {
    case 1: convert_chunks<XT, 1>(s, t); break;
    case 2: convert_chunks<XT, 2>(s, t); break;
    case 3: convert_chunks<XT, 3>(s, t); break;
    case 4: convert_chunks<XT, 4>(s, t); break;
    case 5: convert_chunks<XT, 5>(s, t); break;
    case 6: convert_chunks<XT, 6>(s, t); break;
    case 7: convert_chunks<XT, 7>(s, t); break;
    default: break;
  }
}

// cos/sin of the exact angle l*w (w an fp32 value): the product is exact in
// double; it is reduced by the nearest multiple of 2*pi in double, and the
// fp32 sine/cosine of the reduced angle (|x| <= pi) is taken.
__device__ __forceinline__ void exact_sincos(int l, float w, float& c, float& s) {
  const double a = (double)l * (double)w;
  const double k = rint(a * 0.15915494309189533577);          // a / (2 pi)
  const double red = fma(-k, 6.28318530717958647693, a);
  __sincosf((float)red, &s, &c);
}

// Build W_h = [P | Q] of query head qh for sequence b (fp16, canonical no-swizzle
// K-major layout: row n of W^T, n < 64 -> P, else Q) into Bg, by NT threads
// (thread index t); red holds NT / 32 floats; bar() synchronises the NT threads.
// One pass: thread chunk e = (row i, channels 8kc..8kc+7) computes 8 P and 8 Q
// entries (kc fastest: coalesced U rows), then the block maximum sets the
// power-of-two normalisation eta (largest entries in [2^13, 2^14], fp16's full
// precision; undone in the drain), then fp16 stores.
template <bool QUANT, int NT, typename Bar>
__device__ __forceinline__ void build_w_head(const KParams& p, int b, int qh, const float* qv, uint8_t* Bg, float* red,
                                             int t, Bar bar, float& eta) {
  const starkv_layout& lay = p.lay;
  const int kv = qh / (lay.num_q_heads / lay.num_kv_heads), r = lay.k_rank[kv];
  const int64_t ubase = (int64_t)128 * lay.k_col[kv];
  const __half* scp = QUANT ? p.k_scales + (int64_t)b * lay.k_rank_total + lay.k_col[kv] : nullptr;
  const int nc = r >> 3, nch = 64 * nc;
  constexpr int kPer = (64 * (STARKV_MAX_K_RANK / 8) + NT - 1) / NT;
  float pv[kPer][8], qq[kPer][8];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int e = t + NT * k;
    if (e < nch) {
      const int i = e / nc, kc = e - i * nc;
      const float qa = qv[i], qb = qv[i + 64];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const int c = kc * 8 + cc;
        const float u1 = load_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)i * r + c);
        const float u2 = load_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)(i + 64) * r + c);
        const float sc = QUANT ? __half2float(scp[c]) : 1.f;
        pv[k][cc] = sc * (qa * u1 + qb * u2);
        qq[k][cc] = sc * (qb * u1 - qa * u2);
        amax = fmaxf(amax, fmaxf(fabsf(pv[k][cc]), fabsf(qq[k][cc])));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) red[t >> 5] = amax;
  bar();
  amax = 0.f;
  for (int w = 0; w < NT / 32; ++w) amax = fmaxf(amax, red[w]);
  bar();                                                   // red is reused by the caller
  eta = amax > 0.f ? exp2f(ceilf(log2f(amax)) - 14.f) : 1.f;
  const float inv_eta = 1.f / eta;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int e = t + NT * k;
    if (e < nch) {
      const int i = e / nc, kc = e - i * nc;
      uint32_t op[4], oq[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        __half2 hp = __floats2half2_rn(pv[k][2 * m] * inv_eta, pv[k][2 * m + 1] * inv_eta);
        __half2 hq = __floats2half2_rn(qq[k][2 * m] * inv_eta, qq[k][2 * m + 1] * inv_eta);
        op[m] = *reinterpret_cast<uint32_t*>(&hp);
        oq[m] = *reinterpret_cast<uint32_t*>(&hq);
      }
      *reinterpret_cast<uint4*>(Bg + (i >> 3) * (r * 16) + kc * 128 + (i & 7) * 16) = make_uint4(op[0], op[1], op[2], op[3]);
      *reinterpret_cast<uint4*>(Bg + ((64 + i) >> 3) * (r * 16) + kc * 128 + (i & 7) * 16) = make_uint4(oq[0], oq[1], oq[2], oq[3]);
    }
  }
}

// Pre-pass: W and eta of every (sequence, query head) into the workspace, so that
// the K kernel's prologue is a bulk copy.  grid (Hq, B), 256 threads.
template <bool QUANT>
__global__ void __launch_bounds__(256) k_wprep_kernel(const __grid_constant__ KParams p, uint8_t* wout, float* eout) {
  __shared__ float qv[128];
  __shared__ float red[8];
  const int qh = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const int Hq = p.lay.num_q_heads;
  if (t < 128) qv[t] = load_as_f32(p.q, p.q_dtype, ((int64_t)b * Hq + qh) * 128 + t);
  __syncthreads();
  float eta;
  build_w_head<QUANT, 256>(p, b, qh, qv, wout + ((int64_t)b * Hq + qh) * p.wstride, red, t, [] { __syncthreads(); }, eta);
  if (t == 0) eout[(int64_t)b * Hq + qh] = eta;
}

template <typename XT, bool QUANT, int G>
__global__ void __launch_bounds__(kKThreads, 1) k_logits_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wg = warp >> 2;                      // warpgroup 0..3
  const int split = blockIdx.x, grp = blockIdx.y, b = blockIdx.z;
#ifdef KTRACE_CTA
  const unsigned long long t_start = global_timer_ns();
  __shared__ unsigned long long w_done_s;
#endif
  const starkv_layout& lay = p.lay;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int t_begin = split * p.tps;
  const int t_end = min(p.T, t_begin + p.tps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + 127) / 128 : 0;
  const int NS = p.nstages;
  constexpr int XB = (int)sizeof(XT);

  // ---- shared memory carve-up
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* st_full = bars;                      // [8]  stage landed (tx bytes)
  uint64_t* st_empty = bars + 8;                 // [8]  stage read by the 4 converter warps
  uint64_t* a_full = bars + 16;                  // [4]  A buffer written (4 converter warps)
  uint64_t* a_empty = bars + 20;                 // [4]  A buffer's MMAs retired (commit)
  uint64_t* d_full = bars + 24;                  // [2]  accumulator ready (commit)
  uint64_t* d_empty = bars + 26;                 // [2]  accumulator read by the 8 drain warps
  uint64_t* fin_bar = bars + 28;
  uint64_t* part_full = bars + 29;               // [8]  both halves' partials stored (8 drain warps)
  uint64_t* part_empty = bars + 37;              // [8]  slot read by the job's finaliser warp
  uint64_t* w_bar = bars + 45;                   // W images landed (pre-pass mode)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 512);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 516);
  int* s_nruns = reinterpret_cast<int*>(smem + 520);
  int* s_boff = reinterpret_cast<int*>(smem + 528);           // [4] byte offset of W_g
  int* s_rank = reinterpret_cast<int*>(smem + 544);           // [4] rank of head g
  float* s_epi = reinterpret_cast<float*>(smem + 560);        // [4]
  int* s_run0 = reinterpret_cast<int*>(smem + 576);           // [4] first head of run n
  int* s_runlen = reinterpret_cast<int*>(smem + 592);         // [4] heads in run n
  const uint8_t** s_src = reinterpret_cast<const uint8_t**>(smem + 640);  // [4] latents of (b, kv(g)) at slot 0
  float* s_red = reinterpret_cast<float*>(smem + 704);        // [64]
  float2* s_rot = reinterpret_cast<float2*>(smem + 1024);     // [64] rotation by 128 positions
  float* s_qall = reinterpret_cast<float*>(smem + 1536);      // [4][128]
  float* s_part = reinterpret_cast<float*>(smem + 4096);      // [8][2][128] partial logits of the two halves
  uint8_t* Bsm = smem + kKHeader;
  uint8_t* Ssm = Bsm + (size_t)p.bsum * 256;
  const uint32_t stage_bytes = 128u * p.pitch16max * 16u;

  if (tid == 0) {
    for (int k = 0; k < kKMaxStages; ++k) {
      mbar_init(st_full + k, 1);
      mbar_init(st_empty + k, 4);
    }
    for (int k = 0; k < kKAbufs; ++k) {
      mbar_init(a_full + k, 4);
      mbar_init(a_empty + k, 1);
    }
    for (int k = 0; k < kKAcc; ++k) {
      mbar_init(d_full + k, 1);
      mbar_init(d_empty + k, 8);       // both drain warpgroups
    }
    mbar_init(fin_bar, 1);
    mbar_init(w_bar, 1);
    for (int k = 0; k < kKPartRing; ++k) {
      mbar_init(part_full + k, 8);     // both drain warpgroups
      mbar_init(part_empty + k, 1);    // the finaliser warp of the job
    }
    *s_abort = 0;
    int off = 0, nr = 0;
    for (int g = 0; g < G; ++g) {
      const int kv = (grp * G + g) / qpk;
      s_boff[g] = off;
      s_rank[g] = lay.k_rank[kv];
      s_src[g] = reinterpret_cast<const uint8_t*>(p.k_cache) + (lay.k_offset[kv] + (int64_t)b * lay.k_batch_stride[kv]) * XB;
      off += lay.k_rank[kv] * 256;
      if (g == 0 || kv != (grp * G + g - 1) / qpk) {
        s_run0[nr] = g;
        s_runlen[nr] = 0;
        ++nr;
      }
      ++s_runlen[nr - 1];
    }
    *s_nruns = nr;
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
  const int NR = *s_nruns;
  const int U = ntiles * NR;                     // units of this CTA
  const int J = ntiles * G;                      // jobs of this CTA

  long long* trace = (p.trace && split == 0 && grp == 0 && b < 2) ? p.trace + (int64_t)b * p.trace_jobs * kTrFields
                                                                  : nullptr;
  auto stamp = [&](int j, int f) {
    if (trace && j < p.trace_jobs) trace[(int64_t)j * kTrFields + f] = clock64();
  };
  auto fail = [&](int code) {
    record_error(p.err, code);
    *s_abort = 1;
  };

  if (wg == 0) {
    regs_dec<kKCtlRegs>();
    if (warp == 0) {
      // ============================================================ producer warp
      if (p.wpre && lane == 0) {
        uint32_t wb = 0;
        for (int g = 0; g < G; ++g) wb += (uint32_t)s_rank[g] * 256u;
        mbar_arrive_expect_tx(w_bar, wb);
        for (int g = 0; g < G; ++g)
          bulk_g2s(Bsm + s_boff[g], p.wpre + ((int64_t)b * Hq + grp * G + g) * p.wstride, (uint32_t)s_rank[g] * 256u, w_bar);
      }
      __syncwarp();
      int issued = 0;
      for (int u = 0; u < U; ++u, issued = u) {
        if (*s_abort) break;
        const int s = u % NS;
        if (!mbar_wait(st_empty + s, (uint32_t)(((u / NS) & 1) ^ 1))) { fail(kDevWaitCopy); break; }
        const int t = u / NR, n = u - t * NR;
        const int g0 = s_run0[n], r = s_rank[g0];
        const int t0 = t_begin + t * 128;
        const int nrows = min(128, t_end - t0);
        if (lane == 0) {
          stamp(t * G + g0, kTrLoadIssue);
          const uint32_t bytes = (uint32_t)(nrows * r * XB);
          mbar_arrive_expect_tx(st_full + s, bytes);
          bulk_g2s(Ssm + (size_t)s * stage_bytes, s_src[g0] + (size_t)t0 * r * XB, bytes, st_full + s);
        }
        __syncwarp();
      }
      // every copy this warp issued has landed before the CTA may exit
      if (lane == 0)
        for (int u = max(0, issued - NS); u < issued; ++u)
          if (!mbar_wait(st_full + (u % NS), (uint32_t)((u / NS) & 1))) { fail(kDevWaitCopy); break; }
      __syncwarp();
    } else if (warp == 1) {
      // ============================================================ MMA issuer
      named_bar_sync(1, 416 + 64);               // W matrices built (builders + this warp + finalisers)
      if (p.wpre && lane == 0 && !mbar_wait(w_bar, 0)) fail(kDevWaitCopy);
      if (lane == 0) {
        constexpr uint32_t IDESC = idesc_f16_f32(128, 128);
        // Per-head operands in registers (G is a compile-time constant, so every
        // index below is static): B descriptor, K steps, and whether the head
        // starts a run of heads that share one A buffer (one KV head).
        uint64_t bdesc[G];
        int nk[G];
        bool first[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          bdesc[g] = smem_desc(smem_u32(Bsm + s_boff[g]), 128, (uint32_t)s_rank[g] * 16u);
          nk[g] = s_rank[g] >> 4;
          first[g] = g == 0 || (grp * G + g) / qpk != (grp * G + g - 1) / qpk;
        }
        bool ok = true;
        int u = -1;                                // current unit
        uint32_t a_t = 0;
        for (int t = 0; t < ntiles && ok; ++t) {
          if (*s_abort) break;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int j = t * G + g, db = j & 1;
            if (first[g]) {
              ++u;
              if (!mbar_wait(a_full + (u & (kKAbufs - 1)), (uint32_t)((u / kKAbufs) & 1))) { ok = false; break; }
              a_t = tmem + 256u + (uint32_t)(u & (kKAbufs - 1)) * 64u;
            }
            if (!mbar_wait(d_empty + db, (uint32_t)(((j >> 1) & 1) ^ 1))) { ok = false; break; }
            tc_fence_after();
            stamp(j, kTrMmaIssue);
            const uint32_t d = tmem + (uint32_t)db * 128u;
            mma_f16_ts(d, a_t, bdesc[g], IDESC, 0u);
            for (int kk = 1; kk < nk[g]; ++kk) mma_f16_ts(d, a_t + kk * 8, bdesc[g] + (uint64_t)(kk * 16), IDESC, 1u);
            mma_commit(d_full + db);
            if (g == G - 1 || first[(g + 1) % G]) mma_commit(a_empty + (u & (kKAbufs - 1)));
          }
        }
        if (!ok) fail(kDevWaitMma);
        mma_commit(fin_bar);                     // arrives once every MMA of this thread retired
        if (!mbar_wait(fin_bar, 0)) fail(kDevWaitMma);
      }
      __syncwarp();
    } else {
      // ============================================================ finaliser warps 2, 3
      // Warp 2 + f finishes the jobs j with j % 2 == f: logit = (partial of the low
      // frequencies + partial of the high ones) * scale (+ mask), written to global,
      // and the running maximum per head.  Lane i covers rows i, i+32, i+64, i+96.
      const int f = warp - 2;
      named_bar_sync(1, 416 + 64);               // s_epi ready
      float m_run[G];
#pragma unroll
      for (int g = 0; g < G; ++g) m_run[g] = kNegBig;
      bool ok = true;
      for (int j = f; j < J; j += 2) {
        if (*s_abort) break;
        const int pk = j % kKPartRing;
        if (!mbar_wait(part_full + pk, (uint32_t)((j / kKPartRing) & 1))) { ok = false; break; }
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = s_part[pk * 256 + 32 * q + lane] + s_part[pk * 256 + 128 + 32 * q + lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(part_empty + pk);
        const int tile = j / G, g = j - tile * G;
        const int l0 = t_begin + tile * 128 + lane;
        const float sc = s_epi[g];
        float* dst = p.logits + ((int64_t)b * Hq + grp * G + g) * p.T;
        float mx = kNegBig;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int l = l0 + 32 * q;
          if (l < t_end) {
            float val = v[q] * sc;
            if (p.mask) val = fmaf(p.mask[(int64_t)b * p.T + l], p.mask_scale, val);
            dst[l] = val;
            mx = fmaxf(mx, val);
          }
        }
#pragma unroll
        for (int gg = 0; gg < G; ++gg)
          if (gg == g) m_run[gg] = fmaxf(m_run[gg], mx);
        if (lane == 0) stamp(j, kTrDrainDone);
      }
      if (!ok) fail(kDevWaitMma);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float m = m_run[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_red[g * 8 + f] = m;
      }
    }
  } else {
    // ---- build W_g = [P | Q] (fp16, canonical K-major layout) for each head: 384 threads
    {
      const int bt = tid - 128;
      if (p.wpre) {                                    // W came from the pre-pass (bulk-copied by the producer)
        if (bt < G) s_epi[bt] = p.weta[(int64_t)b * Hq + grp * G + bt] * p.out_scale;
      } else {
        for (int e = bt; e < G * 128; e += 384)
          s_qall[e] = load_as_f32(p.q, p.q_dtype, ((int64_t)b * Hq + grp * G) * 128 + e);
      }
      if (bt < 64) {
        float c, sn;
        exact_sincos(128, p.inv_freq[bt], c, sn);
        s_rot[bt] = make_float2(c, sn);
      }
      named_bar_sync(2, 384);
      for (int g = 0; g < G && !p.wpre; ++g) {
        const int qh = grp * G + g;
        const float* qv = s_qall + g * 128;
        float eta;
        build_w_head<QUANT, 384>(p, b, qh, qv, Bsm + s_boff[g], s_red, bt, [] { named_bar_sync(2, 384); }, eta);
        if (bt == 0) s_epi[g] = eta * p.out_scale;
      }
      fence_proxy_async_smem();
#ifdef KTRACE_CTA
      if (tid == 128) w_done_s = global_timer_ns();
#endif
      named_bar_sync(1, 416 + 64);                       // W ready for the MMA warp (s_epi for the finalisers, s_rot for the drains)
    }

    if (wg == 1) {
      // ============================================================ converter warpgroup
      regs_dec<kKConvRegs>();
      const int ct = tid - 128;                          // token row = TMEM lane
      const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
      // Unit u's TMEM stores complete (and it is handed to the MMA issuer) after the
      // next unit's waits, so the store latency overlaps them.
      int s = 0, sph = 0, n = 0, t = 0;            // stage, its phase, run, tile of unit u
      int prev_s = -1, prev_a = -1, prev_j = 0;
      bool ok = true;
      for (int u = 0; u < U; ++u) {
        if (*s_abort) { ok = false; break; }
        const int a = u & (kKAbufs - 1);
        const int g0 = s_run0[n], r = s_rank[g0];
        const int j = t * G + g0;
        if (!mbar_wait(st_full + s, (uint32_t)sph)) { fail(kDevWaitCopy); ok = false; break; }
        if (ct == 0) stamp(j, kTrConvBegin);
        if (!mbar_wait(a_empty + a, (uint32_t)(((u >> 2) & 1) ^ 1))) { fail(kDevWaitMma); ok = false; break; }
        tc_fence_after();
        if (ct == 0) stamp(j, kTrConvAEmpty);
        const int rc = (r * XB) >> 4;
#ifdef KCONV_PADREAD
        const uint8_t* srow = Ssm + (size_t)s * stage_bytes + (size_t)ct * k_pitch16(r, XB) * 16;
#else
        const uint8_t* srow = Ssm + (size_t)s * stage_bytes + (size_t)ct * r * XB;
#endif
        if (prev_a >= 0) {                         // hand over the previous unit
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(st_empty + prev_s);
            mbar_arrive(a_full + prev_a);
          }
          if (ct == 0) stamp(prev_j, kTrConvDone);
        }
        convert_row<XT>(rc, srow, lane_base + 256u + (uint32_t)a * 64u);
        prev_s = s;
        prev_a = a;
        prev_j = j;
        if (++s == NS) { s = 0; sph ^= 1; }
        if (++n == NR) { n = 0; ++t; }
      }
      if (ok && prev_a >= 0) {
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(st_empty + prev_s);
          mbar_arrive(a_full + prev_a);
        }
        if (ct == 0) stamp(prev_j, kTrConvDone);
      }
    } else {
      // ============================================================ drain: frequency half h
      regs_inc<kKDrainRegs>();
      const int h = wg - 2;
      const int dw = warp & 3;                           // TMEM lane quarter
      const int row = dw * 32 + lane;
      float2 cs_c[16], cs_s[16];                         // cos / sin of frequencies 32h + (2i, 2i+1)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        exact_sincos(t_begin + row, p.inv_freq[32 * h + 2 * i], cs_c[i].x, cs_s[i].x);
        exact_sincos(t_begin + row, p.inv_freq[32 * h + 2 * i + 1], cs_c[i].y, cs_s[i].y);
      }
      const uint32_t lbase = tmem + ((uint32_t)(dw * 32) << 16) + 32u * h;
      bool ok = true;
      int j = 0;
      for (; j < J && ok; ++j) {
        if (*s_abort) { ok = false; break; }
        const int tile = j / G, g = j - tile * G, db = j & 1;
        if (g == 0 && tile > 0) {                        // advance every frequency by 128 positions
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 r0 = s_rot[32 * h + 2 * i], r1 = s_rot[32 * h + 2 * i + 1];
            const float2 c = cs_c[i], sn = cs_s[i];
            cs_c[i] = make_float2(fmaf(c.x, r0.x, -sn.x * r0.y), fmaf(c.y, r1.x, -sn.y * r1.y));
            cs_s[i] = make_float2(fmaf(sn.x, r0.x, c.x * r0.y), fmaf(sn.y, r1.x, c.y * r1.y));
          }
        }
        if (row == 0 && h == 0) stamp(j, kTrDrainWait);
        if (!mbar_wait(d_full + db, (uint32_t)((j >> 1) & 1))) { ok = false; break; }
        tc_fence_after();
        if (row == 0 && h == 0) stamp(j, kTrDrainGot);
        const uint32_t ta = lbase + (uint32_t)db * 128u;
        float va[32], vc[32];
        tmem_ld16x4(ta, ta + 16, ta + 64, ta + 80, va, va + 16, vc, vc + 16);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty + db);      // accumulator free for the MMA of job j + 2
        if (row == 0 && h == 0) stamp(j, kTrDrainLd);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          acc[0] = __ffma2_rn(cs_c[i], make_float2(va[2 * i], va[2 * i + 1]), acc[0]);
          acc[1] = __ffma2_rn(cs_c[i + 1], make_float2(va[2 * i + 2], va[2 * i + 3]), acc[1]);
          acc[2] = __ffma2_rn(cs_s[i], make_float2(vc[2 * i], vc[2 * i + 1]), acc[2]);
          acc[3] = __ffma2_rn(cs_s[i + 1], make_float2(vc[2 * i + 2], vc[2 * i + 3]), acc[3]);
        }
        const float part = ((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y)) + ((acc[2].x + acc[2].y) + (acc[3].x + acc[3].y));
        const int pk = j % kKPartRing;
        if (!mbar_wait(part_empty + pk, (uint32_t)(((j / kKPartRing) & 1) ^ 1))) { ok = false; break; }
        s_part[pk * 256 + 128 * h + row] = part;
        __syncwarp();
        if (lane == 0) mbar_arrive(part_full + pk);
      }
      if (!ok) fail(kDevWaitMma);
    }
  }

  // ---- split statistics and teardown (every MMA retired: the issuer waited fin_bar;
  // every copy landed: the producer waited the last stages)
  tc_fence_before();
  __syncthreads();
#ifdef KTRACE_CTA
  const unsigned long long w_done = w_done_s;
#endif
  if (p.smax && tid < G && !*s_abort) {
    const float M = fmaxf(s_red[tid * 8], s_red[tid * 8 + 1]);
    p.smax[((int64_t)b * Hq + grp * G + tid) * p.nsplit + split] = M;
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#ifdef KTRACE_CTA
  if (tid == 0 && p.trace) {
    long long* ct = p.trace + 2 * p.trace_jobs * kTrFields + 4096 * 8;   // after the V timeline
    const int cid = (b * gridDim.y + grp) * gridDim.x + split;
    ct[cid * 4 + 0] = (long long)t_start;
    ct[cid * 4 + 1] = (long long)global_timer_ns();
    ct[cid * 4 + 2] = (long long)w_done;
    int sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    ct[cid * 4 + 3] = sm;
  }
#endif
}

}  // namespace starkv
