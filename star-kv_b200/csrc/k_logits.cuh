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
// TMEM drain.  The query is folded into W once per step (k_wprep_kernel), so
// neither the keys nor the rotated keys are ever materialised.
//
// k_stream_kernel is persistent: one CTA per SM walks a contiguous range of the
// unit stream (sequence b, KV head kv, 128-token tile), ordered b-major then kv
// then tile.  The ranges are cut by an estimated cost per unit of each KV head
// (HBM bytes, tensor-core and drain time), so that CTAs finish together however
// ragged the ranks are.  A unit carries one job per query head of its KV head.
// 640 threads, roles handing off through mbarriers (every wait bounded):
//   producer warp:   the W images of a new (b, kv) segment and one 1-D bulk copy
//                    per unit (a tile is one contiguous range in HBM) into a
//                    ring of staging slots;
//   converter warpgroups (2, alternate units): thread = token row; reads its
//                    row's 16-byte chunks (conflict-free with the tiled cache
//                    layout), converts to fp16 (int8 codes are exact) and writes
//                    the A operand into a ring of TMEM slots (four of 32
//                    columns when every rank is <= 64, else two of 64);
//   MMA issuers (2, alternate units): per job r/16 tcgen05.mma (A from TMEM,
//                    B = W from shared memory, M=128, N=128, K=16) into
//                    accumulator j mod 3;
//   drain warpgroups (2): each takes half of the 64 RoPE frequencies of every
//                    job (32 cosine and 32 sine columns, two TMEM loads and one
//                    wait, the accumulator released right after), the second
//                    hands its partial sum to the first through shared memory,
//                    which scales, masks, writes the fp32 logit and raises the
//                    head's running maximum (one atomic per warp and job).
// TMEM columns: [0, 384) three accumulators, [384, 512) the A ring.
//
// RoPE angles: each drain thread owns one token row and the cos/sin of its 32
// frequencies; they are exact (double-precision range reduction) at every 16th
// tile of a sequence and advanced tile to tile by the exact rotation through
// 128*w_i.  The values therefore depend only on the token position, not on how
// the stream was cut into CTAs (sharded and unsharded runs agree bit for bit).
// The reference's fp32 product fl(l*w_i) differs from the exact angle by at most
// half an ulp of the angle; for long contexts (ref_angles) the drain applies that
// rounding (first order in the difference, which an FMA gives exactly).
#pragma once
#include "common.cuh"
#include "sm100.cuh"

#include <type_traits>

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
  float* smax;            // (B, Hq) running maximum logit (reset by k_wprep_kernel), or null
  int* err;
  int q_dtype, w_dtype;
  int T, ntiles;          // tokens, 128-token tiles
  int nW, wslot_bytes;    // W slots in shared memory, bytes per slot (qpk W images of rank rmax)
  int nstage, stage_bytes;  // staging slots, bytes per slot (128 rows of rank rmax)
  float out_scale;        // multiplier of q.k (scaling * log2 e for decode)
  float mask_scale;       // multiplier of the mask (log2 e for decode)
  const uint8_t* wpre;    // W of every (sequence, query head) from k_wprep_kernel (stride wstride)
  const float* weta;      // its power-of-two normalisation per (sequence, query head)
  int wstride;            // bytes per (sequence, query head) W image
  int rmax;               // largest K rank of the layout
  int G;                  // KV heads per group: the jobs of a group's tile share one RoPE rotation
  int cost[STARKV_MAX_KV_HEADS];  // scheduling cost of one unit of each KV head
  long long cost_seq;     // sum over KV heads of cost * ntiles: the cost of one sequence
  unsigned long long wait_ns;  // time limit of one device wait
  int ref_angles;         // 1: round each RoPE angle like the reference, fl(l * w_i) in fp32 (long contexts;
                          //    selects the REF instance of k_stream_kernel)
  int skip_unit;          // test hook: the copy of this stream unit is never issued (-1: off)
#ifdef STARKV_KTRACE
  long long* trace;       // diagnostic builds only: clock64 per (job of CTA 0, field)
#endif
};

// Diagnostic timeline (built only with -DSTARKV_KTRACE): clock64 of CTA 0's first
// kKTraceJobs jobs at each hand-off.
#ifdef STARKV_KTRACE
constexpr int kKTraceJobs = 1024, kKTraceFields = 16;
#define KTRACE(job, field)                                                                  \
  do {                                                                                      \
    if (p.trace && blockIdx.x == 0 && (job) < kKTraceJobs) p.trace[(job) * kKTraceFields + (field)] = clock64(); \
  } while (0)
#else
#define KTRACE(job, field) do { } while (0)
#endif

constexpr int kKThreads = 640;
// Register budget per warpgroup after setmaxnreg: control, two converters, two
// drains (48 + 2*64 + 2*152 = 480 <= 5 * 96, the launch budget).
constexpr int kKCtlRegs = 56, kKConvRegs = 56, kKDrainRegs = 152;
constexpr int kKAcc = 3;         // accumulators in TMEM (columns [0, 384))
constexpr int kKASlots = 4;      // A ring slots (at most), TMEM columns [384, 512)
constexpr int kKHeader = 8192;   // barriers, rotations and the partial-sum ring at the start of dynamic smem
constexpr int kKSmemMax = 227 * 1024;
constexpr int kKMaxStages = 32;
constexpr int kKPart = 8;        // partial-sum slots (jobs in flight between the two drain warpgroups)
constexpr int kKAnchor = 16;     // tiles between exact RoPE angles

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

// cos/sin of the exact angle l*w (w an fp32 value): the product is exact in
// double; it is reduced by the nearest multiple of 2*pi in double, and the
// fp32 sine/cosine of the reduced angle (|x| <= pi) is taken.
#ifdef STARKV_SINCOS_NOINLINE
__device__ __noinline__
#else
__device__ __forceinline__
#endif
void exact_sincos(int l, float w, float& c, float& s) {
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

// Pre-pass: W and eta of every (sequence, query head) into the workspace (the K
// kernel's producer bulk-copies them), and the per-head maximum reset.  grid (Hq, B),
// 256 threads.
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
  if (t == 0) {
    eout[(int64_t)b * Hq + qh] = eta;
    if (p.smax) p.smax[(int64_t)b * Hq + qh] = kNegBig;   // the K kernel's running maximum starts here
  }
}

// Units of the stream: segments s = (b, group of G KV heads), ordered b-major;
// within a segment tile-major, then the group's KV heads:
//     u = ((b * ngrp + grp) * ntiles + tile) * G + gk.
// The G * qpk jobs of one tile share the drain's RoPE rotation.  First unit of
// CTA c: the tile where the cumulative cost reaches c / gridDim.x of the total.
__device__ __forceinline__ int k_unit_start(const KParams& p, int c) {
  const int G = p.G, ngrp = p.lay.num_kv_heads / G;
  const long long units = (long long)p.lay.batch * ngrp * p.ntiles * G;
  if (c >= (int)gridDim.x) return (int)units;
  const long long target = (long long)((double)p.cost_seq * p.lay.batch * c / gridDim.x);
  const int b = (int)(target / p.cost_seq);
  long long rem = target - (long long)b * p.cost_seq;
  int grp = 0;
  long long tc = 0;
  for (;; ++grp) {
    tc = 0;
    for (int k = 0; k < G; ++k) tc += p.cost[grp * G + k];
    if (grp + 1 == ngrp || rem < tc * p.ntiles) break;
    rem -= tc * p.ntiles;
  }
  int tile = (int)(rem / tc);
  if (tile >= p.ntiles) tile = p.ntiles - 1;
  return (int)((((long long)b * ngrp + grp) * p.ntiles + tile) * G);
}

// Walks a CTA's units in order; every role keeps its own copy (32-bit unit
// indices: the host checks that they fit).
struct KUnitIter {
  int u, u1;
  int b, grp, tile, gk, kv, seg, ntiles, ngrp, G;
  bool first;                          // first unit of a (b, group) segment in this CTA
  bool tfirst;                         // first unit of a tile in this CTA
  __device__ void init(int u0, int end, int nt, int hkv, int g) {
    u = u0; u1 = end; ntiles = nt; G = g; ngrp = hkv / g; seg = 0; first = tfirst = true;
    const int t = u0 / g;
    gk = u0 - t * g;
    const int s = t / nt;
    tile = t - s * nt;
    b = s / ngrp;
    grp = s - b * ngrp;
    kv = grp * G + gk;
  }
  __device__ bool valid() const { return u < u1; }
  __device__ bool last_of_seg() const { return (tile == ntiles - 1 && gk == G - 1) || u + 1 == u1; }
  __device__ void next() {
    ++u;
    first = tfirst = false;
    if (++gk == G) {
      gk = 0;
      tfirst = true;
      if (++tile == ntiles) {
        tile = 0;
        first = true;
        ++seg;
        if (++grp == ngrp) { grp = 0; ++b; }
      }
    }
    kv = grp * G + gk;
  }
};

// Store n (multiple of 4, <= 32) consecutive 32-bit TMEM columns of this warp's
// lanes (register offsets stay compile-time constants).
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t* o, int n) {
  switch (n) {
    case 32: tmem_st32(taddr, o); break;
    case 28: tmem_st16(taddr, o); tmem_st8(taddr + 16, o + 16); tmem_st4(taddr + 24, o + 24); break;
    case 24: tmem_st16(taddr, o); tmem_st8(taddr + 16, o + 16); break;
    case 20: tmem_st16(taddr, o); tmem_st4(taddr + 16, o + 16); break;
    case 16: tmem_st16(taddr, o); break;
    case 12: tmem_st8(taddr, o); tmem_st4(taddr + 8, o + 8); break;
    case 8: tmem_st8(taddr, o); break;
    default: tmem_st4(taddr, o); break;
  }
}

// Convert up to NCH staged 16-byte chunks of one row (chunk stride cs) into
// packed fp16 pairs o[] (cols_per_chunk(XT) columns per chunk).
template <typename XT, int NCH>
__device__ __forceinline__ void k_convert_piece(const uint8_t* src, int cs, int nch, uint32_t* o) {
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (c < nch) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + c * cs);
      if constexpr (sizeof(XT) == 1) {
        cvt8_i8(w.x, w.y, o + 8 * c);
        cvt8_i8(w.z, w.w, o + 8 * c + 4);
      } else if constexpr (std::is_same<XT, __half>::value) {
        o[4 * c] = w.x; o[4 * c + 1] = w.y; o[4 * c + 2] = w.z; o[4 * c + 3] = w.w;
      } else if constexpr (std::is_same<XT, __nv_bfloat16>::value) {
        const uint32_t in[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __half2 h = __floats2half2_rn(__uint_as_float(in[k] << 16), __uint_as_float(in[k] & 0xFFFF0000u));
          o[4 * c + k] = *reinterpret_cast<uint32_t*>(&h);
        }
      } else {
        __half2 h0 = __floats2half2_rn(__uint_as_float(w.x), __uint_as_float(w.y));
        __half2 h1 = __floats2half2_rn(__uint_as_float(w.z), __uint_as_float(w.w));
        o[2 * c] = *reinterpret_cast<uint32_t*>(&h0);
        o[2 * c + 1] = *reinterpret_cast<uint32_t*>(&h1);
      }
    }
  }
}

template <typename XT, bool REF>
__global__ void __launch_bounds__(kKThreads, 1) k_stream_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wg = __shfl_sync(0xffffffffu, warp >> 2, 0);   // warpgroup 0..4 (warp-uniform)
  const starkv_layout& lay = p.lay;
  const int Hq = lay.num_q_heads, Hkv = lay.num_kv_heads, qpk = Hq / Hkv;
  const int G = p.G, GJ = G * qpk;                         // KV heads per group, jobs per tile
  constexpr int XB = (int)sizeof(XT);
  constexpr int CPC = 8 / XB;                              // TMEM columns (fp16 pairs) per 16-byte chunk
  constexpr int PCH = (32 / CPC) < 8 ? (32 / CPC) : 8;     // chunks per conversion piece (<= 32 columns)
  const bool tiled = lay.k_tiled != 0;
  // A ring: four 32-column slots when every rank is <= 64 (r fp16 per row = r / 2
  // columns), else two of 64.  Unit i takes slot i % nAs; since the converter
  // warpgroups, and the issuers, alternate units, every slot is always written
  // by the same warpgroup and read by the same issuer, so each waits its slot's
  // phases strictly in order.
  const int nAs = p.rmax <= 64 ? 4 : 2, aW = 128 / nAs;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* st_full = bars;                   // [32] staging slot landed (tx bytes)
  uint64_t* st_empty = bars + 32;             // [32] staging slot read (4 converter warps)
  uint64_t* a_full = bars + 64;               // [4]  A slot written (4 converter warps)
  uint64_t* a_empty = bars + 68;              // [4]  A slot's MMAs retired (commit)
  uint64_t* d_full = bars + 72;               // [3]  accumulator ready (commit)
  uint64_t* d_empty = bars + 75;              // [3]  accumulator read (8 drain warps)
  uint64_t* p_full = bars + 78;               // [8]  partial sum of a job written (4 warps of the other drain)
  uint64_t* w_full = bars + 86;               // [2]  W slot landed (tx bytes)
  uint64_t* w_empty = bars + 88;              // [2]  W slot's MMAs retired (one commit per issuer)
  uint64_t* fin_bar = bars + 90;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 1024);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 1028);
  int* s_range = reinterpret_cast<int*>(smem + 1040);               // [2] unit range of this CTA
  float* s_esc = reinterpret_cast<float*>(smem + 1088);             // [2][8] logit scale of each job of the segment
  float2* s_w = reinterpret_cast<float2*>(smem + 1280);             // [32] inverse frequencies (2i, 2i+1)
  float4* s_rot = reinterpret_cast<float4*>(smem + 1536);           // [32] rotation by one tile
  float* s_part = reinterpret_cast<float*>(smem + 2048);            // [8][128]
  uint8_t* Wsm = smem + kKHeader;
  uint8_t* Ssm = Wsm + (size_t)p.nW * p.wslot_bytes;

  if (tid == 0) {
    for (int k = 0; k < kKMaxStages; ++k) {
      mbar_init(st_full + k, 1);
      mbar_init(st_empty + k, 4);
    }
    for (int k = 0; k < kKASlots; ++k) {
      mbar_init(a_full + k, 4);
      mbar_init(a_empty + k, 1);
    }
    for (int k = 0; k < kKAcc; ++k) {
      mbar_init(d_full + k, 1);
      mbar_init(d_empty + k, 8);
    }
    for (int k = 0; k < kKPart; ++k) mbar_init(p_full + k, 4);
    for (int k = 0; k < 2; ++k) {
      mbar_init(w_full + k, 1);
      mbar_init(w_empty + k, 2);
    }
    mbar_init(fin_bar, 2);
    *s_abort = 0;
    s_range[0] = k_unit_start(p, blockIdx.x);
    s_range[1] = k_unit_start(p, blockIdx.x + 1);
    fence_mbar_init();
  }
  if (warp == 2) {                                          // rotation of frequency pair (2i, 2i+1) by 128 positions
    const int i = lane;
    float c0, s0, c1, s1;
    exact_sincos(128, p.inv_freq[2 * i], c0, s0);
    exact_sincos(128, p.inv_freq[2 * i + 1], c1, s1);
    s_rot[i] = make_float4(c0, c1, s0, s1);
    s_w[i] = make_float2(p.inv_freq[2 * i], p.inv_freq[2 * i + 1]);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int u0 = s_range[0], u1 = s_range[1];
#ifdef STARKV_KTRACE
  if (p.trace && tid == 0) {
    p.trace[kKTraceJobs * kKTraceFields + blockIdx.x * 4 + 0] = (long long)global_timer_ns();
    p.trace[kKTraceJobs * kKTraceFields + blockIdx.x * 4 + 2] = u1 - u0;
  }
#endif
  const unsigned long long wlim = p.wait_ns;
  auto fail_at = [&](int code, int line) {
    record_error(p.err, code);
    *s_abort = 1;
#ifdef STARKV_KTRACE
    if (p.trace)
      atomicCAS(reinterpret_cast<unsigned long long*>(p.trace + kKTraceJobs * kKTraceFields + blockIdx.x * 4 + 3), 0ull,
                (unsigned long long)line);
#else
    (void)line;
#endif
  };
#define fail(code) fail_at(code, __LINE__)
  const int NS = p.nstage;

  if (wg == 0) {
    regs_dec<kKCtlRegs>();
    if (warp == 0) {
      // ============================================================ producer
      if (lane == 0) {
        KUnitIter it;
        it.init(u0, u1, p.ntiles, Hkv, G);
        int i = 0, nseg = 0;
        for (; it.valid(); it.next(), ++i) {
          if (*s_abort) break;
          const int r = lay.k_rank[it.kv], R = r * XB;
          if (it.first) {                                   // the segment's W images, job order
            const int k = it.seg, ws = k % p.nW;
            nseg = k + 1;
            if (k >= p.nW && !mbar_wait(w_empty + ws, (uint32_t)(((k / p.nW) & 1) ^ 1), wlim)) { fail(kDevWaitMma); break; }
            uint32_t wb = 0;
            for (int gk = 0; gk < G; ++gk) wb += (uint32_t)(qpk * lay.k_rank[it.grp * G + gk] * 256);
            mbar_arrive_expect_tx(w_full + ws, wb);
            uint32_t off = 0;
            for (int gk = 0; gk < G; ++gk) {
              const int kv = it.grp * G + gk, rk = lay.k_rank[kv];
              for (int g = 0; g < qpk; ++g) {
                bulk_g2s(Wsm + (size_t)ws * p.wslot_bytes + off, p.wpre + ((int64_t)it.b * Hq + kv * qpk + g) * p.wstride,
                         (uint32_t)(rk * 256), w_full + ws);
                off += (uint32_t)(rk * 256);
              }
            }
          }
          const int s = i % NS;
          if (!mbar_wait(st_empty + s, (uint32_t)(((i / NS) & 1) ^ 1), wlim)) { fail(kDevWaitCopy); break; }
          if (it.u == p.skip_unit) continue;                   // test hook: this stage never lands
          const int t0 = it.tile * 128;
          const uint32_t bytes = (uint32_t)((tiled ? 128 : min(128, p.T - t0)) * R);
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.k_cache) +
                               (lay.k_offset[it.kv] + (int64_t)it.b * lay.k_batch_stride[it.kv]) * XB + (int64_t)t0 * R;
          mbar_arrive_expect_tx(st_full + s, bytes);
          bulk_g2s(Ssm + (size_t)s * p.stage_bytes, src, bytes, st_full + s);
          KTRACE(i, 0);
        }
        // every copy issued has landed before the CTA may exit (each wait bounded;
        // a stage that was never issued only costs its time limit)
        for (int k = max(0, i - NS); k < i; ++k)
          if (!(u0 + k == p.skip_unit) && !mbar_wait(st_full + k % NS, (uint32_t)((k / NS) & 1), wlim))
            fail(kDevWaitCopy);
        for (int k = max(0, nseg - p.nW); k < nseg; ++k)
          if (!mbar_wait(w_full + k % p.nW, (uint32_t)((k / p.nW) & 1), wlim)) fail(kDevWaitCopy);
      }
      __syncwarp();
    } else if (warp == 1 || warp == 2) {
      // ============================================================ MMA issuers
      // Issuer iw takes the units i with i % 2 == iw (one thread issues a
      // tcgen05.mma about as fast as the tensor core retires one, so two keep it
      // busy); both walk every unit to follow the job, A-ring and W offsets.
      // (With several jobs per unit one issuer keeps the tensor core busy, and
      // two could run one accumulator phase ahead of the drains.)
      const int iw = warp - 1;
      const int NI = qpk == 1 ? 2 : 1;                       // issuers
      if (lane == 0 && iw < NI) {
        constexpr uint32_t IDESC = idesc_f16_f32(128, 128);
        KUnitIter it;
        it.init(u0, u1, p.ntiles, Hkv, G);
        int j = 0;
        uint32_t woff = 0;                                  // byte offset of this KV head's W images in the slot
        bool ok = true;
        for (int i = 0; it.valid() && ok; it.next(), ++i) {
          if (*s_abort) break;
          const int r = lay.k_rank[it.kv];
          const int ws = it.seg % p.nW;
          const int as = i % nAs;                              // A slot of unit i, used for the (i / nAs)-th time
          if (it.tfirst) {
            woff = 0;
            for (int gk = 0; gk < it.gk; ++gk) woff += (uint32_t)(qpk * lay.k_rank[it.grp * G + gk] * 256);
          }
          if (i % NI == iw) {
            if (it.first && !mbar_wait(w_full + ws, (uint32_t)((it.seg / p.nW) & 1), wlim)) { ok = false; break; }
            if (!mbar_wait(a_full + as, (uint32_t)((i / nAs) & 1), wlim)) { ok = false; break; }
            tc_fence_after();
            KTRACE(j, 4);
            const uint32_t acol = 384u + (uint32_t)(as * aW);
            for (int g = 0; g < qpk; ++g) {
              const int jj = j + g;
              if (jj >= kKAcc && !mbar_wait(d_empty + jj % kKAcc, (uint32_t)(((jj / kKAcc) - 1) & 1), wlim)) { ok = false; break; }
              tc_fence_after();
              KTRACE(jj, 5);
              const uint64_t bdesc = smem_desc(smem_u32(Wsm + (size_t)ws * p.wslot_bytes + woff + g * r * 256), 128,
                                               (uint32_t)r * 16u);
              const uint32_t d = tmem + (uint32_t)(jj % kKAcc) * 128u;
              for (int kk = 0; kk < (r >> 4); ++kk)
                mma_f16_ts(d, tmem + acol + 8u * kk, bdesc + (uint64_t)(kk * 16), IDESC, kk ? 1u : 0u);
              mma_commit(d_full + jj % kKAcc);
              KTRACE(jj, 6);
            }
            if (!ok) break;
            mma_commit(a_empty + as);
          }
          if (it.last_of_seg())                             // every issuer: the slot is free once all retired
            for (int k = NI; k <= 2; ++k) mma_commit(w_empty + ws);
          woff += (uint32_t)(qpk * r * 256);
          j += qpk;
        }
        if (!ok) fail(kDevWaitMma);
        mma_commit(fin_bar);                     // arrives once every MMA of this thread retired
        if (NI == 1) mma_commit(fin_bar);
        if (!mbar_wait(fin_bar, 0, wlim)) fail(kDevWaitMma);
      }
      __syncwarp();
    }
  } else if (wg <= 2) {
    // ============================================================ converter warpgroups
    // Warpgroup cw takes the units i with i % 2 == cw; both walk every unit to
    // follow the A ring.
    regs_dec<kKConvRegs>();
    const int cw = wg - 1;
    const int row = tid - 128 * wg;                          // token row = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    KUnitIter it;
    it.init(u0, u1, p.ntiles, Hkv, G);
    for (int i = 0; it.valid(); it.next(), ++i) {
      const int r = lay.k_rank[it.kv];
      const int as = i % nAs;
      if ((i & 1) == cw) {
        if (*s_abort) break;
        const int s = i % NS;
        if (!mbar_wait(st_full + s, (uint32_t)((i / NS) & 1), wlim)) { fail(kDevWaitCopy); break; }
        if (row == 0) KTRACE(i, 1);
        const int R = r * XB, nch = R >> 4;
        const int cs = tiled ? 2048 : 16;
        const uint8_t* srow = Ssm + (size_t)s * p.stage_bytes + (tiled ? row * 16 : row * R);
        const uint32_t acol = 384u + (uint32_t)(as * aW);
        // the first piece is converted before the A slots are free (its latency
        // overlaps the wait), the rest after
        uint32_t o[32];
        k_convert_piece<XT, PCH>(srow, cs, min(PCH, nch), o);
        if (!mbar_wait(a_empty + as, (uint32_t)(((i / nAs) & 1) ^ 1), wlim)) { fail(kDevWaitMma); break; }
        tc_fence_after();
        if (row == 0) KTRACE(i, 2);
        tmem_st_cols(lane_base + acol, o, min(PCH, nch) * CPC);
        for (int c0 = PCH; c0 < nch; c0 += PCH) {
          const int n = min(PCH, nch - c0);
          k_convert_piece<XT, PCH>(srow + c0 * cs, cs, n, o);
          tmem_st_cols(lane_base + acol + (uint32_t)(c0 * CPC), o, n * CPC);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(st_empty + s);            // the stage is read: back to the producer
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
          mbar_arrive(a_full + as);
        if (lane == 0) KTRACE(i, (row >> 5) == 0 ? 3 : 12 + (row >> 5));
      }
    }
  } else {
    // ============================================================ drain warpgroups
    // Half h = wg - 3 takes frequencies [32h, 32h + 32) of every job: cosine
    // columns [32h, 32h + 32) and sine columns [64 + 32h, 96 + 32h).  The job's
    // epilogue (sum of the halves, scale, mask, logit, running maximum) is done by
    // half (j & 1); the other hands its partial sum over in shared memory.
    regs_inc<kKDrainRegs>();
    const int h = wg - 3;
    const int dw = warp & 3;
    const int row = dw * 32 + lane;
    const uint32_t lbase = tmem + ((uint32_t)(dw * 32) << 16);
    float2 cc[16], ss[16];                                   // cos / sin of frequencies (32h + 2i, 32h + 2i + 1)
    float m_run[8];                                          // running maximum of each job of the segment
    KUnitIter it;
    it.init(u0, u1, p.ntiles, Hkv, G);
    int j = 0;
    bool ok = true;
    float madd = 0.f, lpos = 0.f;
    bool live = false;
    int l = 0;
    auto flush_max = [&](int b, int kv0) {                   // the segment's maxima -> per-head global maximum
      if (!p.smax) return;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e < GJ) {
          float m = m_run[e];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0 && m > kNegBig) atomic_max_float(p.smax + (int64_t)b * Hq + kv0 * qpk + e, m);
        }
        m_run[e] = kNegBig;
      }
    };
#pragma unroll
    for (int e = 0; e < 8; ++e) m_run[e] = kNegBig;
    int seg_b = it.b, seg_kv0 = it.grp * G;
    for (; it.valid() && ok; it.next()) {
      if (*s_abort) break;
      if (it.first) {
        if (it.seg > 0) flush_max(seg_b, seg_kv0);
        seg_b = it.b;
        seg_kv0 = it.grp * G;
        named_bar_sync(2 + h, 128);                          // this half's reads of the previous scales are done
        if (row < GJ) s_esc[h * 8 + row] = p.weta[(int64_t)it.b * Hq + seg_kv0 * qpk + row] * p.out_scale;
        named_bar_sync(2 + h, 128);
      }
      if (it.tfirst) {
        // ---- RoPE angles of this tile's token rows
        const int tile = it.tile;
        int nrot = 1;                                        // rotations by one tile still to apply
        if (it.first || (tile % kKAnchor) == 0) {
          const int a = tile - tile % kKAnchor;
          const int pos = a * 128 + row;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 w = s_w[16 * h + i];
            exact_sincos(pos, w.x, cc[i].x, ss[i].x);
            exact_sincos(pos, w.y, cc[i].y, ss[i].y);
            asm volatile("" ::: "memory");                   // one frequency pair at a time (register pressure)
          }
          nrot = tile - a;
        }
#pragma unroll 1
        for (int k = 0; k < nrot; ++k) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float4 rt = s_rot[16 * h + i];
            const float2 rc = make_float2(rt.x, rt.y), rs = make_float2(rt.z, rt.w);
            const float2 c = cc[i], sn = ss[i];
            const float2 uu = __fmul2_rn(sn, rs), vv = __fmul2_rn(c, rs);
            cc[i] = __ffma2_rn(c, rc, make_float2(-uu.x, -uu.y));
            ss[i] = __ffma2_rn(sn, rc, vv);
            asm volatile("" ::: "memory");                   // keep each constant's load beside its use
          }
        }
        l = tile * 128 + row;
        lpos = (float)l;
        live = l < p.T;
        madd = (p.mask && live) ? p.mask[(int64_t)it.b * p.T + l] * p.mask_scale : 0.f;
      }
#pragma unroll 1
      for (int g = 0; g < qpk; ++g, ++j) {
        const int e = it.gk * qpk + g;                       // job within the segment's tile
        const int acc = j % kKAcc;
        if (!mbar_wait(d_full + acc, (uint32_t)((j / kKAcc) & 1), wlim)) { ok = false; break; }
        tc_fence_after();
        if (row == 0) KTRACE(j, 7 + h);
        float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
        if constexpr (REF) {
          // The reference's angle is fl(l * w) = l * w - e with e = fma(l, w, -fl(l * w))
          // exact; cos / sin of it to first order in e (|e| <= half an ulp of the angle):
          // c + s e and s - c e.
          const float2 lf = make_float2(lpos, lpos), nlf = make_float2(-lpos, -lpos);
          {
            float v[32];
            tmem_ld32(lbase + (uint32_t)acc * 128u + 32u * h, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 w = s_w[16 * h + i];
              const float2 er = __ffma2_rn(lf, w, __fmul2_rn(nlf, w));
              const float2 c = __ffma2_rn(ss[i], er, cc[i]);
              a0 = __ffma2_rn(c, make_float2(v[2 * i], v[2 * i + 1]), a0);
            }
          }
          {
            float v[32];
            tmem_ld32(lbase + (uint32_t)acc * 128u + 64u + 32u * h, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty + acc);      // accumulator free for the MMA of job j + 3
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 w = s_w[16 * h + i];
              const float2 ne = __ffma2_rn(nlf, w, __fmul2_rn(lf, w));
              const float2 sn = __ffma2_rn(cc[i], ne, ss[i]);
              a1 = __ffma2_rn(sn, make_float2(v[2 * i], v[2 * i + 1]), a1);
            }
          }
        } else {
          {
            float v[32];
            tmem_ld32(lbase + (uint32_t)acc * 128u + 32u * h, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) a0 = __ffma2_rn(cc[i], make_float2(v[2 * i], v[2 * i + 1]), a0);
          }
          {
            float v[32];
            tmem_ld32(lbase + (uint32_t)acc * 128u + 64u + 32u * h, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty + acc);      // accumulator free for the MMA of job j + 3
#pragma unroll
            for (int i = 0; i < 16; ++i) a1 = __ffma2_rn(ss[i], make_float2(v[2 * i], v[2 * i + 1]), a1);
          }
        }
        const float part = (a0.x + a0.y) + (a1.x + a1.y);
        if (row == 0 && h == 0) KTRACE(j, 9);
        const int ps = j % kKPart;
        if ((j & 1) != h) {
          s_part[ps * 128 + row] = part;
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full + ps);
          if (row == 0) KTRACE(j, 10);
        } else {
          if (!mbar_wait(p_full + ps, (uint32_t)((j / kKPart) & 1), wlim)) { ok = false; break; }
          if (row == 0) KTRACE(j, 11);
          const float val = fmaf(part + s_part[ps * 128 + row], s_esc[h * 8 + e], madd);
          if (live) {
            p.logits[((int64_t)it.b * Hq + it.kv * qpk + g) * p.T + l] = val;
#pragma unroll
            for (int k = 0; k < 8; ++k)
              if (k == e) m_run[k] = fmaxf(m_run[k], val);
          }
          if (row == 0) KTRACE(j, 12);
        }
      }
    }
    if (ok && !*s_abort) flush_max(seg_b, seg_kv0);
    if (!ok) fail(kDevWaitMma);
  }

  // ---- teardown (every MMA retired: the issuers waited fin_bar; every copy landed:
  // the producer waited the last stages)
  tc_fence_before();
  __syncthreads();
#ifdef STARKV_KTRACE
  if (p.trace && tid == 0) p.trace[kKTraceJobs * kKTraceFields + blockIdx.x * 4 + 1] = (long long)global_timer_ns();
#endif
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#undef fail
}

}  // namespace starkv
