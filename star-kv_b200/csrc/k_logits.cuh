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
// CTA = (sequence b, group of G query heads, split of the group's tokens; each
// group has its own split count, chosen on the host to balance ragged ranks), 640 threads, one
// CTA per SM (it owns the 512 TMEM columns).  A "unit" is one 128-token tile of
// one KV head (the G heads form runs of heads that share a KV head); a "job" is
// one (tile, query head) pair.  Roles, handing off through mbarriers (every wait
// bounded):
//   producer warp:   one 1-D bulk copy per unit (its rows are one contiguous
//                    block in HBM) into a ring of tile slots in shared memory;
//   converter warpgroups (2, alternate units): thread = token row; converts its
//                    staged row (its 16-byte chunks 16 bytes apart in the
//                    row-major layout, 2 KiB apart in the tiled one, where a
//                    warp's reads are conflict-free) to fp16 (int8 codes are exact in fp16) into
//                    registers, releases the stage, waits for its own A buffer in
//                    TMEM and writes it with wide tcgen05.st — the A operand never
//                    touches shared memory;
//   MMA issuers (warps 1 and 2 for one-job units, else warp 1): per job r/16
//                    tcgen05.mma (A from TMEM, B = W_g from shared memory, M=128,
//                    N=128, K=16) into accumulator j mod 3;
//   drain warpgroups (2, alternate tiles): thread = token row; eight 16-column
//                    tcgen05.ld of the accumulator (released right after), the
//                    RoPE-weighted sum over all 64 frequencies (packed fp32x2 FMA),
//                    scale, mask, the logit to global and a running maximum per
//                    head — the split maximum the V kernel's softmax starts from
//                    (the V kernel forms the exponentials and their sums itself).
// TMEM columns: [0, 384) three accumulators, [384, 512) two A buffers of 64
// columns (r <= 128 fp16 values per row).
//
// RoPE angles: each drain thread owns one token row; it starts from cos/sin of
// l*w_i for the first token of its first tile and advances by the exact rotation
// through 256*w_i to its next tile (fp32, packed FMAs, shared by the G heads of
// the tile).  The angles are the exact l*w_i; the reference's fp32 product
// fl(l*w_i) differs from them by at most half an ulp of the angle.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace starkv {

constexpr int kKMaxGroups = 64;  // head groups per layer (Hq / G)

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
  int T, nsplit, tps;     // tokens, split stride of smax (the most splits of any group), unused
  int ngroups, splits_seq;                   // head groups; CTAs per sequence (sum of gsplit)
  int gsplit[kKMaxGroups];                   // sequence splits of each head group
  int G, rmax, bsum;      // heads per CTA, max rank, max per-group rank sum (W matrices in smem)
  int stage_total;        // bytes of the staging ring
  float out_scale;        // multiplier of q.k (scaling * log2 e for decode)
  float mask_scale;       // multiplier of the mask (log2 e for decode)
  const uint8_t* wpre;    // W of every (sequence, query head) from k_wprep_kernel (stride wstride), or null:
  const float* weta;      //   then the CTA builds its W itself; eta of every (sequence, query head)
  int wstride;            // bytes per (sequence, query head) W image
  unsigned long long wait_ns;  // time limit of one device wait
  int skip_unit;          // test hook: the first CTA never issues this unit's copy (-1: off)
#ifdef STARKV_KTRACE
  long long* trace;       // diagnostic builds only: clock64 per (job of CTA 0, field), CTA start / end
#endif
};
#ifdef STARKV_KTRACE
#define KTRACE(j, f)                                                                                  \
  do {                                                                                                \
    if (p.trace && blockIdx.x == 0 && (j) < 1024) p.trace[(j) * 16 + (f)] = clock64();               \
  } while (0)
#else
#define KTRACE(j, f) do { } while (0)
#endif

constexpr int kKThreads = 640;
// Register budget per warpgroup after setmaxnreg: control, two converters, two
// drains (32 + 2*64 + 2*160 = 480 <= 5 * 96, the launch budget).
constexpr int kKCtlRegs = 32, kKConvRegs = 64, kKDrainRegs = 160;
static_assert(kKCtlRegs + 2 * kKConvRegs + 2 * kKDrainRegs <= 5 * (65536 / kKThreads / 8 * 8),
              "setmaxnreg split above the registers the CTA is launched with");
constexpr int kKAbufs = 2;       // A buffers in TMEM (columns [384, 512)), one per converter warpgroup
constexpr int kKAcc = 3;         // accumulators in TMEM (columns [0, 384))
constexpr int kKHeader = 12288;  // barriers / scratch / partial-logit ring at the start of dynamic smem
constexpr int kKSmemMax = 227 * 1024;

// Staging ring: a CTA's units are staged row-major (one bulk copy of 128 * R
// contiguous bytes, R = r * element size) into tile slots; a tile slot holds the
// units of every run of one 128-token tile back to back, and the ring has as
// many tile slots as shared memory allows (at most kKMaxSlots unit slots).
constexpr int kKMaxSlots = 32;

// Staging bytes next to the W matrices of one CTA (one CTA per SM).
__host__ __device__ inline long k_stage_total(int bsum) {
  return ((long)kKSmemMax - kKHeader - (long)bsum * 256) & ~15L;
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
__device__ __forceinline__ void convert_chunks(const uint8_t* srow, int cs, uint32_t taddr) {
  uint4 w[N];
#pragma unroll
  for (int c = 0; c < N; ++c) w[c] = *reinterpret_cast<const uint4*>(srow + cs * c);
#pragma unroll
  for (int c = 0; c < N; ++c) cvt_store<XT>(w[c], taddr + c * k_cols_per_chunk<XT>());
}

// int8 row of RC chunks: loads, conversions into registers, then the fewest wide
// TMEM stores (x32 / x16 / x8 columns), at most 4 chunks (32 columns) at a time.
template <int N>
__device__ __forceinline__ void convert_row_i8(const uint8_t* srow, int cs, uint32_t taddr) {
  if constexpr (N > 4) {
    convert_row_i8<4>(srow, cs, taddr);
    convert_row_i8<N - 4>(srow + 4 * cs, cs, taddr + 32);
  } else {
    uint4 w[N];
#pragma unroll
    for (int c = 0; c < N; ++c) w[c] = *reinterpret_cast<const uint4*>(srow + cs * c);
    uint32_t o[8 * N];
#pragma unroll
    for (int c = 0; c < N; ++c) {
      cvt8_i8(w[c].x, w[c].y, o + 8 * c);
      cvt8_i8(w[c].z, w[c].w, o + 8 * c + 4);
    }
    if constexpr (N == 4) {
      tmem_st32(taddr, o);
    } else {
      int col = 0;
      if constexpr (N >= 2) {
        tmem_st16(taddr, o);
        col = 16;
      }
      if constexpr (N & 1) tmem_st8(taddr + col, o + col);
    }
  }
}

// int8 row of RC <= 6 chunks converted into registers (two chunks loaded at a
// time), and the stores of such a row (fewest wide tcgen05.st): the conversion
// can run before the row's A buffer is free, the stores after.
template <int RC>
__device__ __forceinline__ void load_cvt_i8(const uint8_t* srow, int cs, uint32_t* o) {
#pragma unroll
  for (int c = 0; c < RC; c += 2) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(srow + cs * c);
    uint4 w1 = make_uint4(0u, 0u, 0u, 0u);
    if (c + 1 < RC) w1 = *reinterpret_cast<const uint4*>(srow + cs * (c + 1));
    cvt8_i8(w0.x, w0.y, o + 8 * c);
    cvt8_i8(w0.z, w0.w, o + 8 * c + 4);
    if (c + 1 < RC) {
      cvt8_i8(w1.x, w1.y, o + 8 * c + 8);
      cvt8_i8(w1.z, w1.w, o + 8 * c + 12);
    }
  }
}
template <int RC>
__device__ __forceinline__ void store_row_i8(uint32_t taddr, const uint32_t* o) {
  int col = 0;
#pragma unroll
  for (; col + 32 <= 8 * RC; col += 32) tmem_st32(taddr + col, o + col);
  if constexpr ((8 * RC) % 32 >= 16) {
    tmem_st16(taddr + col, o + col);
    col += 16;
  }
  if constexpr ((8 * RC) % 16 >= 8) tmem_st8(taddr + col, o + col);
}

// Convert, release the stage, wait for the A buffer, store: RC <= 6 int8 chunks.
template <int RC, typename Release, typename WaitA>
__device__ __forceinline__ bool convert_ahead_i8(const uint8_t* srow, int cs, uint32_t taddr, Release release,
                                                 WaitA wait_a) {
  uint32_t o[8 * RC];
  load_cvt_i8<RC>(srow, cs, o);
  release();
  if (!wait_a()) return false;
  store_row_i8<RC>(taddr, o);
  return true;
}

// Convert a staged row of rc chunks into TMEM: int8 rows in one piece, other
// element types in groups of 8 chunks, then the rest.
template <typename XT>
__device__ __forceinline__ void convert_row(int rc, const uint8_t* srow, int cs, uint32_t taddr) {
  if constexpr (sizeof(XT) == 1) {
    switch (rc) {
      case 1: convert_row_i8<1>(srow, cs, taddr); return;
      case 2: convert_row_i8<2>(srow, cs, taddr); return;
      case 3: convert_row_i8<3>(srow, cs, taddr); return;
      case 4: convert_row_i8<4>(srow, cs, taddr); return;
      case 5: convert_row_i8<5>(srow, cs, taddr); return;
      case 6: convert_row_i8<6>(srow, cs, taddr); return;
      case 7: convert_row_i8<7>(srow, cs, taddr); return;
      case 8: convert_row_i8<8>(srow, cs, taddr); return;
      default: break;
    }
  }
  int c = 0;
  for (; c + 8 <= rc; c += 8) convert_chunks<XT, 8>(srow + cs * c, cs, taddr + c * k_cols_per_chunk<XT>());
  const uint8_t* sr = srow + cs * c;
  const uint32_t t = taddr + c * k_cols_per_chunk<XT>();
  switch (rc - c) {
    case 1: convert_chunks<XT, 1>(sr, cs, t); break;
    case 2: convert_chunks<XT, 2>(sr, cs, t); break;
    case 3: convert_chunks<XT, 3>(sr, cs, t); break;
    case 4: convert_chunks<XT, 4>(sr, cs, t); break;
    case 5: convert_chunks<XT, 5>(sr, cs, t); break;
    case 6: convert_chunks<XT, 6>(sr, cs, t); break;
    case 7: convert_chunks<XT, 7>(sr, cs, t); break;
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

// Elements [i, i + 8) of a dtype-tagged array as float: one 16-byte load for
// 16-bit types when the address is 16-byte aligned, else element by element.
__device__ __forceinline__ void load8_as_f32(const void* p, int dtype, int64_t i, float* out) {
  if (dtype != STARKV_F32) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p) + i;
    if ((reinterpret_cast<uintptr_t>(q) & 15) == 0) {
      const uint4 w = *reinterpret_cast<const uint4*>(q);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (dtype == STARKV_F16) {
          const __half2 h = *reinterpret_cast<const __half2*>(&ws[e]);
          out[2 * e] = __low2float(h);
          out[2 * e + 1] = __high2float(h);
        } else {
          out[2 * e] = __uint_as_float(ws[e] << 16);
          out[2 * e + 1] = __uint_as_float(ws[e] & 0xFFFF0000u);
        }
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) out[e] = load_as_f32(p, dtype, i + e);
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
      float u1v[8], u2v[8], scv[8];                       // 8 consecutive channels: 16-byte loads where possible
      load8_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)i * r + kc * 8, u1v);
      load8_as_f32(p.k_u, p.w_dtype, ubase + (int64_t)(i + 64) * r + kc * 8, u2v);
      if (QUANT) load8_as_f32(scp, STARKV_F16, kc * 8, scv);
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const float u1 = u1v[cc], u2 = u2v[cc];
        const float sc = QUANT ? scv[cc] : 1.f;
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
  if (p.smax)                                      // splits a group does not use stay at "minus infinity"
    for (int k = t; k < p.nsplit; k += 256) p.smax[((int64_t)b * Hq + qh) * p.nsplit + k] = kNegBig;
}

template <typename XT, bool QUANT, int G>
__global__ void __launch_bounds__(kKThreads, 1) k_logits_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wg = __shfl_sync(0xffffffffu, warp >> 2, 0);   // warpgroup 0..4 (warp-uniform)
  // CTA = (sequence b, head group, split of that group); groups have their own
  // split counts (cost-balanced on the host), CTAs are numbered b-major.
  const int b = blockIdx.x / p.splits_seq;
  int grp = 0, split = blockIdx.x - b * p.splits_seq;
  while (split >= p.gsplit[grp]) split -= p.gsplit[grp++];
  const int gns = p.gsplit[grp];
  const int gtps = (((p.T + 127) / 128 + gns - 1) / gns) * 128;
  const starkv_layout& lay = p.lay;
  const int Hq = lay.num_q_heads, qpk = Hq / lay.num_kv_heads;
  const int t_begin = split * gtps;
  const int t_end = min(p.T, t_begin + gtps);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + 127) / 128 : 0;
  constexpr int XB = (int)sizeof(XT);
  const bool tiled = lay.k_tiled != 0;                   // tiles stored as 16-byte column chunks (starkv.h)
  const unsigned long long wlim = p.wait_ns;

  // ---- shared memory carve-up
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 8192);
  uint64_t* st_full = bars;                      // [32] unit slot landed (tx bytes)
  uint64_t* st_empty = bars + 32;                // [32] unit slot read by the 4 converter warps
  uint64_t* a_full = bars + 64;                  // [2]  A buffer written (4 converter warps)
  uint64_t* a_empty = bars + 80;                 // [2]  A buffer's MMAs retired (commit)
  uint64_t* d_full = bars + 96;                  // [6G] job slot j % 6G: accumulator j % 3 ready (commit)
  uint64_t* d_empty = bars + 120;                // [6G] job slot j % 6G: accumulator read by the job's 4 drain warps
  uint64_t* fin_bar = bars + 144;
  uint64_t* w_bar = bars + 145;                  // W images landed (pre-pass mode)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 512);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 516);
  int* s_nruns = reinterpret_cast<int*>(smem + 520);
  int* s_boff = reinterpret_cast<int*>(smem + 528);           // [4] byte offset of W_g
  int* s_rank = reinterpret_cast<int*>(smem + 544);           // [4] rank of head g
  const uint8_t** s_src = reinterpret_cast<const uint8_t**>(smem + 640);  // [4] latents of (b, kv(g)) at slot 0
  float* s_epi = reinterpret_cast<float*>(smem + 560);        // [4]
  int* s_run0 = reinterpret_cast<int*>(smem + 576);           // [4] first head of run n
  int* s_runlen = reinterpret_cast<int*>(smem + 592);         // [4] heads in run n
  float* s_red = reinterpret_cast<float*>(smem + 704);        // [64]
  float4* s_rot4 = reinterpret_cast<float4*>(smem + 4096);    // [32] rotation by 256 positions per frequency pair (cos.xy, sin.xy)
  float* s_qall = reinterpret_cast<float*>(smem + 1536);      // [4][128]
  uint8_t* Bsm = smem + kKHeader;
  uint8_t* Ssm = Bsm + (size_t)p.bsum * 256;
  int* s_runoff = reinterpret_cast<int*>(smem + 4608);        // [4] byte offset of run n in a tile slot
  int* s_ring = reinterpret_cast<int*>(smem + 4624);          // [2] tile slots, bytes per tile slot

  if (tid == 0) {
    for (int k = 0; k < kKMaxSlots; ++k) {
      mbar_init(st_full + k, 1);
      mbar_init(st_empty + k, 4);
    }
    for (int k = 0; k < kKAbufs; ++k) {
      mbar_init(a_full + k, 4);
      mbar_init(a_empty + k, 1);
    }
    for (int k = 0; k < 6 * G; ++k) {
      mbar_init(d_full + k, 1);
      mbar_init(d_empty + k, 4);       // the drain warpgroup of the job
    }
    mbar_init(w_bar, 1);
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
    mbar_init(fin_bar, nr == G ? 2 : 1);       // one arrival per MMA issuer
    int tb = 0;
    for (int n = 0; n < nr; ++n) {
      s_runoff[n] = tb;
      tb += 128 * s_rank[s_run0[n]] * XB;
    }
    int nt = p.stage_total / tb;
    if (nt > kKMaxSlots / nr) nt = kKMaxSlots / nr;
    s_ring[0] = nt;                              // >= 2 (checked on the host)
    s_ring[1] = tb;
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
#ifdef STARKV_KTRACE
  if (tid == 0 && p.trace && blockIdx.x < 1024) p.trace[16384 + blockIdx.x * 2] = (long long)global_timer_ns();
#endif
  const int NR = *s_nruns;
  const int NT = s_ring[0];                      // tile slots in the ring
  const int TB = s_ring[1];                      // bytes per tile slot
  const int U = ntiles * NR;                     // units of this CTA

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
      if (lane == 0) {
        int t = 0, n = 0;                          // tile and run of unit u
        for (int u = 0; u < U; ++u, issued = u) {
          if (*s_abort) break;
          const int ts = t % NT, slot = ts * NR + n;
          if (!mbar_wait(st_empty + slot, (uint32_t)(((t / NT) & 1) ^ 1), wlim)) { fail(kDevWaitCopy); break; }
          const int g0 = s_run0[n], R = s_rank[g0] * XB;
          const int t0 = t_begin + t * 128;
          const uint32_t bytes = (uint32_t)((tiled ? 128 : min(128, t_end - t0)) * R);
          const bool skip = u == p.skip_unit && blockIdx.x == 0;
          if (!skip) {                               // (test hook: a skipped stage never lands)
            mbar_arrive_expect_tx(st_full + slot, bytes);
            bulk_g2s(Ssm + (size_t)ts * TB + s_runoff[n], s_src[g0] + (size_t)t0 * R, bytes, st_full + slot);
            KTRACE(u, 0);
          }
          if (++n == NR) { n = 0; ++t; }
        }
        // every copy issued has landed before the CTA may exit
        for (int u = max(0, issued - NT * NR); u < issued; ++u) {
          const int tt = u / NR, slot = (tt % NT) * NR + (u - tt * NR);
          if (u == p.skip_unit && blockIdx.x == 0) continue;
          if (!mbar_wait(st_full + slot, (uint32_t)((tt / NT) & 1), wlim)) fail(kDevWaitCopy);   // each bounded
        }
      }
      __syncwarp();
    } else if (warp == 1 || warp == 2) {
      // ============================================================ MMA issuers
      // When every query head of the group has its own KV head (one job per unit),
      // warps 1 and 2 issue the units of parity 0 and 1 (the bookkeeping of one
      // overlaps the MMAs of the other); otherwise warp 1 issues every unit.  Job j
      // accumulates into accumulator j % 3 and signals job slot j % 6G (the jobs of
      // one slot share their issuer and their drain warpgroup, so each slot's phases
      // are waited in order); before reusing accumulator j % 3 the issuer waits for
      // job j - 3 to be drained (slot (j - 3) % 6G, at most one phase behind: this
      // issuer waited for job j - 3 - 6G before it issued job j - 6G).
      named_bar_sync(1, 512 + 96);               // W matrices built (builders + warps 1-3)
      const int NI = (NR == G) ? 2 : 1;          // issuers
      const int iw = warp - 1;
      if (iw < NI && lane == 0) {
        if (p.wpre && !mbar_wait(w_bar, 0, wlim)) fail(kDevWaitCopy);
        constexpr uint32_t IDESC = idesc_f16_f32(128, 128);
        bool ok = true;
        int t = 0, n = iw;                         // tile and run of unit u
        if (n >= NR) { n -= NR; ++t; }
        for (int u = iw; u < U && ok; u += NI) {
          if (!mbar_wait(a_full + (u & 1), (uint32_t)((u >> 1) & 1), wlim)) { ok = false; break; }
          KTRACE(u, 4);
          const uint32_t a_t = tmem + 384u + (uint32_t)(u & 1) * 64u;
          const int g0 = s_run0[n], len = s_runlen[n];
          for (int k = 0; k < len; ++k) {
            const int g = g0 + k, j = t * G + g;
            if (j >= kKAcc) {
              const int jp = j - kKAcc;
              if (!mbar_wait(d_empty + jp % (6 * G), (uint32_t)((jp / (6 * G)) & 1), wlim)) { ok = false; break; }
            }
            KTRACE(j, 5);
            tc_fence_after();
            const int r = s_rank[g];
            const uint64_t bdesc = smem_desc(smem_u32(Bsm + s_boff[g]), 128, (uint32_t)r * 16u);
            const uint32_t d = tmem + (uint32_t)(j % kKAcc) * 128u;
            mma_f16_ts(d, a_t, bdesc, IDESC, 0u);
            for (int kk = 1; kk < (r >> 4); ++kk) mma_f16_ts(d, a_t + kk * 8, bdesc + (uint64_t)(kk * 16), IDESC, 1u);
            mma_commit(d_full + j % (6 * G));
            KTRACE(j, 6);
          }
          mma_commit(a_empty + (u & 1));
          n += NI;
          while (n >= NR) { n -= NR; ++t; }
        }
        if (!ok) fail(kDevWaitMma);
        mma_commit(fin_bar);                     // arrives once every MMA of this thread retired
        if (!mbar_wait(fin_bar, 0, wlim)) fail(kDevWaitMma);
      }
      __syncwarp();
    } else {
      // warp 3: no role after the prologue barrier
      named_bar_sync(1, 512 + 96);
    }
  } else {
    // ---- build W_g = [P | Q] (fp16, canonical K-major layout) for each head: 512 threads
    {
      const int bt = tid - 128;
      if (p.wpre) {                                    // W came from the pre-pass (bulk-copied by the producer)
        if (bt < G) s_epi[bt] = p.weta[(int64_t)b * Hq + grp * G + bt] * p.out_scale;
      } else {
        for (int e = bt; e < G * 128; e += 512)
          s_qall[e] = load_as_f32(p.q, p.q_dtype, ((int64_t)b * Hq + grp * G) * 128 + e);
      }
      named_bar_sync(2, 512);
      if (bt >= 64 && bt < 96) {                       // rotation of the pair (2i, 2i + 1) by 256 positions: cos, sin
        const int i = bt - 64;
        float c0, s0, c1, s1;
        exact_sincos(256, p.inv_freq[2 * i], c0, s0);
        exact_sincos(256, p.inv_freq[2 * i + 1], c1, s1);
        s_rot4[i] = make_float4(c0, c1, s0, s1);
      }
      for (int g = 0; g < G && !p.wpre; ++g) {
        const int qh = grp * G + g;
        const float* qv = s_qall + g * 128;
        float eta;
        build_w_head<QUANT, 512>(p, b, qh, qv, Bsm + s_boff[g], s_red, bt, [] { named_bar_sync(2, 512); }, eta);
        if (bt == 0) s_epi[g] = eta * p.out_scale;
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 512 + 96);                       // W ready for the MMA warp (s_epi, s_rot4 for the drains)
    }

    if (wg <= 2) {
      // ============================================================ converter warpgroups
      // Warpgroup c = wg - 1 converts the units u with u % 2 == c into A buffer c.
      regs_dec<kKConvRegs>();
      const int cw = wg - 1;
      const int ct = tid - 128 * wg;                     // token row = TMEM lane
      const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
      // Each unit is handed to the MMA issuer as soon as its TMEM stores complete
      // (this warpgroup's next unit waits for the same A buffer to drain).
      int n = cw, t = 0;                           // run, tile of unit u
      while (n >= NR) { n -= NR; ++t; }
      for (int u = cw; u < U; u += 2) {
        if (*s_abort) break;
        const int g0 = s_run0[n], r = s_rank[g0];
        const int ts = t % NT, s = ts * NR + n;
        if (!mbar_wait(st_full + s, (uint32_t)((t / NT) & 1), wlim)) { fail(kDevWaitCopy); break; }
        if (ct == 0) KTRACE(u, 1);
        const int rc = (r * XB) >> 4;
        const int cs = tiled ? 2048 : 16;            // bytes between a row's 16-byte chunks
        const uint8_t* srow = Ssm + (size_t)ts * TB + s_runoff[n] + (size_t)ct * (tiled ? 16 : r * XB);
        const uint32_t taddr = lane_base + 384u + (uint32_t)cw * 64u;
        auto release = [&] {                       // the stage is read: hand it back to the producer
          __syncwarp();
          if (lane == 0) mbar_arrive(st_empty + s);
        };
        auto wait_a = [&]() -> bool {              // the A buffer's previous MMAs retired
          if (!mbar_wait(a_empty + cw, (uint32_t)(((u >> 1) & 1) ^ 1), wlim)) { fail(kDevWaitMma); return false; }
          tc_fence_after();
          if (ct == 0) KTRACE(u, 2);
          return true;
        };
        bool okc = true;
        if constexpr (XB == 1) {
          switch (rc) {
            case 1: okc = convert_ahead_i8<1>(srow, cs, taddr, release, wait_a); break;
            case 2: okc = convert_ahead_i8<2>(srow, cs, taddr, release, wait_a); break;
            case 3: okc = convert_ahead_i8<3>(srow, cs, taddr, release, wait_a); break;
            case 4: okc = convert_ahead_i8<4>(srow, cs, taddr, release, wait_a); break;
            case 5: okc = convert_ahead_i8<5>(srow, cs, taddr, release, wait_a); break;
            case 6: okc = convert_ahead_i8<6>(srow, cs, taddr, release, wait_a); break;
            default:
              okc = wait_a();
              if (okc) convert_row<XT>(rc, srow, cs, taddr);
              release();
              break;
          }
        } else {
          okc = wait_a();
          if (okc) convert_row<XT>(rc, srow, cs, taddr);
          release();
        }
        if (!okc) break;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + cw);
        if (ct == 0) KTRACE(u, 3);
        n += 2;
        while (n >= NR) { n -= NR; ++t; }
      }
    } else {
      // ============================================================ drain warpgroups
      // Warpgroup w = wg - 3 takes every job of the tiles t with t % 2 == w.  Per
      // job: thread = token row (TMEM lane) with cos / sin of all 64 frequencies at
      // its token in registers (advanced by 256 positions per tile of its own with
      // packed fp32x2 rotations), eight 16-column TMEM loads, packed fp32x2 FMAs,
      // then scale, mask, the logit to HBM and the running maximum per head.
      regs_inc<kKDrainRegs>();
      const int w2 = wg - 3;
      const int dw = warp & 3;                           // TMEM lane quarter
      const int row = dw * 32 + lane;
      float2 cs_c[32], cs_s[32];                         // cos / sin of frequencies (2i, 2i+1)
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        exact_sincos(t_begin + 128 * w2 + row, p.inv_freq[2 * i], cs_c[i].x, cs_s[i].x);
        exact_sincos(t_begin + 128 * w2 + row, p.inv_freq[2 * i + 1], cs_c[i].y, cs_s[i].y);
      }
      float m_run[G];
#pragma unroll
      for (int g = 0; g < G; ++g) m_run[g] = kNegBig;
      const uint32_t lbase = tmem + ((uint32_t)(dw * 32) << 16);
      float* const lg_base = p.logits + ((int64_t)b * Hq + grp * G) * p.T + t_begin + row;
      bool ok = true;
      for (int tile = w2; tile < ntiles && ok; tile += 2) {
        if (*s_abort) { ok = false; break; }
        if (tile > w2) {                                 // advance every frequency by 256 positions
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float4 r = s_rot4[i];
            const float2 rc = make_float2(r.x, r.y), rs = make_float2(r.z, r.w);
            const float2 c = cs_c[i], sn = cs_s[i];
            const float2 u = __fmul2_rn(sn, rs), v = __fmul2_rn(c, rs);
            cs_c[i] = __ffma2_rn(c, rc, make_float2(-u.x, -u.y));
            cs_s[i] = __ffma2_rn(sn, rc, v);
            asm volatile("" ::: "memory");               // keep each constant's load beside its use (no hoisting)
          }
        }
#pragma unroll 1
        for (int g = 0; g < G; ++g) {
          const int j = tile * G + g;
          const int db = j % kKAcc, ds = j % (6 * G);    // accumulator, job slot
          // the epilogue's operands first, so that their latency overlaps the waits
          const int l = t_begin + tile * 128 + row;
          const bool live = l < t_end;
          const float esc = s_epi[g];
          const float madd = (p.mask && live) ? p.mask[(int64_t)b * p.T + l] * p.mask_scale : 0.f;
          float* const dst = lg_base + (int64_t)g * p.T + tile * 128;
          if (!mbar_wait(d_full + ds, (uint32_t)((j / (6 * G)) & 1), wlim)) { ok = false; break; }
          if (row == 0) KTRACE(j, 7);
          tc_fence_after();
          const uint32_t ta = lbase + (uint32_t)db * 128u;
          float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
          for (int q = 0; q < 8; ++q) {                  // columns [16q, 16q + 16): q < 4 cosine part, else sine part
            float v[16];
            tmem_ld16(ta + 16u * q, v);
            if (q == 7) {                                // accumulator free for the MMA of job j + kKAcc
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(d_empty + ds);
              if (row == 0) KTRACE(j, 8);
            }
            const int f0 = (q & 3) * 8;                  // first frequency pair of this block
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              if (q < 4) {
                acc0 = __ffma2_rn(cs_c[f0 + i], make_float2(v[2 * i], v[2 * i + 1]), acc0);
                acc1 = __ffma2_rn(cs_c[f0 + i + 1], make_float2(v[2 * i + 2], v[2 * i + 3]), acc1);
              } else {
                acc0 = __ffma2_rn(cs_s[f0 + i], make_float2(v[2 * i], v[2 * i + 1]), acc0);
                acc1 = __ffma2_rn(cs_s[f0 + i + 1], make_float2(v[2 * i + 2], v[2 * i + 3]), acc1);
              }
            }
          }
          const float sum = (acc0.x + acc0.y) + (acc1.x + acc1.y);
          if (live) {
            const float val = fmaf(sum, esc, madd);
            *dst = val;
#pragma unroll
            for (int gg = 0; gg < G; ++gg)
              if (gg == g) m_run[gg] = fmaxf(m_run[gg], val);
          }
          if (row == 0) KTRACE(j, 9);
        }
      }
      if (!ok) fail(kDevWaitMma);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float m = m_run[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_red[g * 8 + w2 * 4 + dw] = m;
      }
    }
  }

  // ---- split statistics and teardown (every MMA retired: the issuer waited fin_bar;
  // every copy landed: the producer waited the last stages)
  tc_fence_before();
  __syncthreads();
  if (p.smax && tid < G && !*s_abort) {
    float M = s_red[tid * 8];
#pragma unroll
    for (int k = 1; k < 8; ++k) M = fmaxf(M, s_red[tid * 8 + k]);
    p.smax[((int64_t)b * Hq + grp * G + tid) * p.nsplit + split] = M;
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#ifdef STARKV_KTRACE
  if (tid == 0 && p.trace && blockIdx.x < 1024) p.trace[16384 + blockIdx.x * 2 + 1] = (long long)global_timer_ns();
#endif
}

}  // namespace starkv
