// prefill.cuh — prompt (prefill) attention on the 5th-generation tensor cores.
//
// The reference's prompt path rebuilds full K / V from the latents
// (K = RoPE(X_k U_k^T), V = X_v U_v^T) and runs causal SDPA over them
// (model.py:429-449, LlamaLoRaAttention_headwise.py:100-116).  This kernel is the
// attention half of that: causal flash attention with the online softmax, K / V
// of the query head's KV head (GQA by index), q / k / v / out as strided
// (B, H, T, 128) views so that the projections' (B, T, H, 128) tensors are read
// and written in place.
//
// CTA = (pair of 128-query tiles 2i and 2i+1, query head, sequence), heaviest
// pairs first, 352 threads, one CTA per SM (all 512 TMEM columns):
//   * warp 9 lane 0: TMA loads of the two Q tiles and of a two-stage ring of
//     (K_j, V_j) tiles shared by both query tiles, each tile two 64-channel x
//     128-row boxes in the 128-byte swizzled layout — the canonical K-major
//     layout for Q and K and the MN-major one for V (channels along N, tokens
//     along K: no transposition).  Rows past the sequence end are zero-filled.
//   * warp 8 lane 0 issues S_X(j) = Q_X K_j^T, warp 10 lane 0 issues
//     O_X += P_X(j) V_j (8 tcgen05.mma each, M = N = 128, K = 16; A = P from TMEM).
//   * warps 0-3 (query tile 0) and 4-7 (tile 1), one thread per query row
//     holding the whole S row: row maximum (lazy: the running maximum moves only
//     when a tile exceeds it by more than 2^2, then O and l of that row are
//     rescaled in TMEM), weights x = S * scale - m in fp32 and 2^x by a packed
//     fp16 MUFU ex2 for half of the pairs and a packed fp32x2 polynomial on the
//     FMA pipe for the other half, written as 16-bit P over the S row in TMEM.
// Every wait is bounded (mbarriers only, no named barriers); a wait that runs
// out records an error code, sets the CTA's abort flag and the roles leave
// their loops.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace starkv {

constexpr int kPfTile = 128;                    // queries per query tile and keys per step
constexpr int kPfTileBytes = 128 * 128 * 2;     // one 128 x 128 16-bit tile
constexpr int kPfHeader = 3072;                 // barriers, TMEM address, abort flag

struct PrefillParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t q_stride[3];     // elements: batch, head, token (the 128 channels are contiguous)
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int batch, num_q_heads, num_kv_heads, num_tokens, n_qtiles;
  int out_dtype;
  float scale_log2;        // softmax scale * log2(e)
  int* err;                // device error word (nullable)
  unsigned long long wait_ns;
  long long* trace;        // diagnostic builds (STARKV_PFTRACE): CTA 0 timeline, else null
  uint32_t v_lbo, v_sbo;   // V operand descriptor strides (MN-major, 128-byte swizzle)
};

#ifdef STARKV_PFTRACE
#define PFTRACE(j, f)                                                                           \
  do {                                                                                          \
    if (p.trace && blockIdx.x == 0 && (j) < 512) p.trace[(j) * 16 + (f)] = clock64();            \
  } while (0)
#else
#define PFTRACE(j, f) do { } while (0)
#endif

// Instruction descriptor, kind::f16 with A = B = 16-bit type T, D = f32, A K-major,
// B K-major (b_mn = false) or MN-major (b_mn = true), M = N = 128.
template <typename T>
__host__ __device__ constexpr uint32_t idesc_pf(bool b_mn) {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(128 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed 2^x of two fp16 values (one MUFU instruction for both).
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// 2^x of two fp32 values on the FMA pipe (packed fp32x2 arithmetic), for x <= 2:
// n = round(x) through the 1.5 * 2^23 rounding constant, f = x - n in [-0.5, 0.5],
// 2^f ~ 1 + f (c1 + f (c2 + f c3)) (coefficients fitted here to the relative
// error on [-0.5, 0.5]: |rel err| <= 1.02e-4, below half an ulp of fp16), and n
// added to the exponent field.  x is clamped at -127 (the result is then below
// the fp16 range and rounds to 0).
__device__ __forceinline__ float2 poly_exp2x2(float2 x) {
  constexpr float kRound = 12582912.f;             // 1.5 * 2^23, bit pattern 0x4B400000
  x = make_float2(fmaxf(x.x, -127.f), fmaxf(x.y, -127.f));
  const float2 r = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(r, make_float2(-kRound, -kRound));
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 q = __ffma2_rn(f, make_float2(0.05500900f, 0.05500900f), make_float2(0.24221100f, 0.24221100f));
  q = __ffma2_rn(f, q, make_float2(0.69328290f, 0.69328290f));
  q = __ffma2_rn(f, q, make_float2(1.f, 1.f));
  const uint32_t ex = (uint32_t)(__float_as_int(r.x) - 0x4B400000) << 23;
  const uint32_t ey = (uint32_t)(__float_as_int(r.y) - 0x4B400000) << 23;
  return make_float2(__uint_as_float(__float_as_uint(q.x) + ex), __uint_as_float(__float_as_uint(q.y) + ey));
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Shared-memory matrix descriptor for the 128-byte swizzled canonical layouts
// (rows of 128 bytes, 16-byte chunks XOR-ed with row % 8, 8-row atoms of 1024
// bytes at 1024-byte aligned addresses).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return smem_desc(saddr, lbo, sbo) | (2ull << 61);
}

// 4-D tiled TMA load (no multicast) completing on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// Two query tiles per CTA.  CTA = (pair of 128-query tiles 2i, 2i+1, query
// head, sequence): both tiles share every K / V tile load and the tensor core
// alternates between them.  TMEM: tile X in {0, 1} owns columns 256X..256X+255
// — S_j (fp32, 128 columns) at +0, overwritten by P_j (16-bit pairs, 64
// columns) once its row has been read, and the output accumulator at +128.
// Warp 8 issues S = Q K^T, warp 10 issues O += P V (two issuing threads: one
// thread issues an M = N = 128 MMA only every ~120 cycles); S_X(j+1) overwrites
// P_X(j), so its issuer first waits for P_X(j) V_j to complete, which also
// makes O_X safe for the softmax to rescale once it sees S_X(j+1).  Warp 9
// loads tiles by TMA.  Warps 0-3 own tile 0, warps 4-7 tile 1, one thread per
// query row holding the whole S row: no cross-thread exchange.
constexpr int kPf2Threads = 352;
constexpr int kPf2Stages = 2;
constexpr size_t kPf2Smem = kPfHeader + (2 + 2 * kPf2Stages) * (size_t)kPfTileBytes;

template <typename T>
__global__ void __launch_bounds__(kPf2Threads, 1)
    prefill_attn2_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;     // [2]
  uint64_t* kv_empty = bar + 3;    // [2]
  uint64_t* s_full = bar + 5;      // [2]: per query tile
  uint64_t* p_full = bar + 7;      // [2]: per query tile
  uint64_t* pv_done = bar + 9;     // [2]: per query tile, its latest P V complete
  uint64_t* s_done = bar + 11;     // S issuer's MMAs complete (teardown)
  uint64_t* o_done = bar + 12;     // P V issuer's MMAs complete (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 256);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 260);
  uint8_t* Qs = smem + kPfHeader;                  // tile X at X * kPfTileBytes
  uint8_t* KVs = Qs + 2 * kPfTileBytes;            // stage s: K at 2s, V at 2s+1

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int per = p.num_q_heads * p.batch;
  const int npairs = (p.n_qtiles + 1) >> 1;
  const int pi = npairs - 1 - (int)blockIdx.x / per;   // heaviest pairs first
  const int h = ((int)blockIdx.x % per) % p.num_q_heads;
  const int b = ((int)blockIdx.x % per) / p.num_q_heads;
  const int kvh = h / (p.num_q_heads / p.num_kv_heads);
  const int q0 = 2 * pi;                           // query tiles q0, q0 + 1
  const bool has1 = q0 + 1 < p.n_qtiles;
  const int n0 = q0 + 1;                           // key tiles of query tile 0
  const int nk = has1 ? q0 + 2 : n0;               // key tiles the CTA loads
  const unsigned long long lim = p.wait_ns;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
      mbar_init(s_full + s, 1);
      mbar_init(p_full + s, 128);
      mbar_init(pv_done + s, 1);
    }
    mbar_init(s_done, 1);
    mbar_init(o_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint64_t* bar_, uint32_t parity, int code) -> bool {
    if (*s_abort) return false;
    if (mbar_wait(bar_, parity, lim)) return true;
    record_error(p.err, code);
    *s_abort = 1;
    return false;
  };

  if (warp == 9) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, (has1 ? 2 : 1) * kPfTileBytes);
      for (int x = 0; x < (has1 ? 2 : 1); ++x) {
        tma_load_4d(Qs + x * kPfTileBytes, &tm_q, 0, (q0 + x) * kPfTile, h, b, q_full);
        tma_load_4d(Qs + x * kPfTileBytes + kPfTileBytes / 2, &tm_q, 64, (q0 + x) * kPfTile, h, b, q_full);
      }
      for (int j = 0; j < nk; ++j) {
        const int st = j % kPf2Stages;
        if (j >= kPf2Stages && !wait(kv_empty + st, ((j / kPf2Stages) - 1) & 1, kDevWaitMma)) break;
        uint8_t* kt = KVs + (size_t)st * 2 * kPfTileBytes;
        uint8_t* vt = kt + kPfTileBytes;
        mbar_arrive_expect_tx(kv_full + st, 2 * kPfTileBytes);
        tma_load_4d(kt, &tm_k, 0, j * kPfTile, kvh, b, kv_full + st);
        tma_load_4d(kt + kPfTileBytes / 2, &tm_k, 64, j * kPfTile, kvh, b, kv_full + st);
        tma_load_4d(vt, &tm_v, 0, j * kPfTile, kvh, b, kv_full + st);
        tma_load_4d(vt + kPfTileBytes / 2, &tm_v, 64, j * kPfTile, kvh, b, kv_full + st);
      }
    }
    __syncwarp();
  } else if (warp == 8) {
    // ------------------------------------------------------------ S = Q K^T
    if (lane == 0) {
      constexpr uint32_t IS = idesc_pf<T>(false);
      bool ok = wait(q_full, 0, kDevWaitCopy);
      for (int j = 0; ok && j < nk; ++j) {
        if (!wait(kv_full + (j % kPf2Stages), (j / kPf2Stages) & 1, kDevWaitCopy)) break;
        const uint32_t kb = smem_u32(KVs + (size_t)(j % kPf2Stages) * 2 * kPfTileBytes);
        for (int x = 0; x < (has1 ? 2 : 1); ++x) {
          if (j >= (x ? nk : n0)) continue;
          // S_x(j) overwrites P_x(j-1): wait for P_x(j-1) V_{j-1} to complete
          if (j >= 1 && !wait(pv_done + x, (j - 1) & 1, kDevWaitMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qa = smem_u32(Qs + x * kPfTileBytes);
          const uint32_t d = tmem + (uint32_t)x * 256;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16_ss(d, smem_desc_sw128(qa + (kk >> 2) * (kPfTileBytes / 2) + (kk & 3) * 32, 16, 1024),
                       smem_desc_sw128(kb + (kk >> 2) * (kPfTileBytes / 2) + (kk & 3) * 32, 16, 1024), IS,
                       kk > 0 ? 1u : 0u);
          mma_commit(s_full + x);
          PFTRACE(j, 4 + x);
        }
      }
      mma_commit(s_done);
      mbar_wait(s_done, 0, lim);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------------------ O += P V
    if (lane == 0) {
      constexpr uint32_t IO = idesc_pf<T>(true);
      bool ok = true;
      for (int j = 0; ok && j < nk; ++j) {
        const uint32_t vb = smem_u32(KVs + (size_t)(j % kPf2Stages) * 2 * kPfTileBytes + kPfTileBytes);
        for (int x = 0; x < (has1 ? 2 : 1); ++x) {
          if (j >= (x ? nk : n0)) continue;
          if (!wait(p_full + x, j & 1, kDevWaitMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t pa = tmem + (uint32_t)x * 256;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16_ts(pa + 128, pa + kk * 8, smem_desc_sw128(vb + kk * 2048, p.v_lbo, p.v_sbo), IO,
                       (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(pv_done + x);
          PFTRACE(j, 6 + x);
        }
        // S_x(j) finished before the softmax released P_x(j): the stage is free after these P V
        if (ok) mma_commit(kv_empty + (j % kPf2Stages));
      }
      mma_commit(o_done);
      mbar_wait(o_done, 0, lim);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax
    const int x = warp >> 2;                       // query tile of this warpgroup
    const int row = tid & 127;                     // TMEM lane == query row
    const int qt = q0 + x;
    const int nx = x ? nk : n0;
    const int qpos = qt * kPfTile + row;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sa = tmem + lane_base + (uint32_t)x * 256;    // S_j, then P_j
    const uint32_t o_col = sa + 128;
    float m_run = kNegBig, l_run = 0.f;
    const float sl2 = p.scale_log2;
    constexpr float kLazy = 2.f;                   // log2 of the largest weight (fp16 ex2 input precision)
    bool ok = (x == 0 || has1);
    for (int j = 0; ok && j < nx; ++j) {
      if (!__all_sync(0xffffffffu, wait(s_full + x, j & 1, kDevWaitMma))) { ok = false; break; }
      if (row == 0 && x == 0) PFTRACE(j, 8);
      tc_fence_after();
      float sv[128];
      tmem_ld32x2(sa, sa + 32, sv, sv + 32);
      tmem_ld32x2(sa + 64, sa + 96, sv + 64, sv + 96);
      const bool diag = (j == qt);
      const int kmax = diag ? row : 127;
      float mq[4] = {kNegBig, kNegBig, kNegBig, kNegBig};
      if (!diag) {
#pragma unroll
        for (int i = 0; i < 128; i += 8) {
          mq[0] = max3(mq[0], sv[i], sv[i + 1]);
          mq[1] = max3(mq[1], sv[i + 2], sv[i + 3]);
          mq[2] = max3(mq[2], sv[i + 4], sv[i + 5]);
          mq[3] = max3(mq[3], sv[i + 6], sv[i + 7]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) mq[i & 3] = (i <= kmax) ? fmaxf(mq[i & 3], sv[i]) : mq[i & 3];
      }
      const float mt = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
      if (j == 0) {
        m_run = mt;
      } else {
        const bool need = mt > m_run + kLazy;
        float alpha = 1.f;
        if (need) {
          alpha = fast_exp2(m_run - mt);
          m_run = mt;
          l_run *= alpha;
        }
        // O_X holds P_0 V_0 + ... + P_{j-1} V_{j-1}: S_X(j) was issued after they completed
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float v[16];
            tmem_ld16(o_col + c * 16, v);
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(v[i] * alpha);
            tmem_st16(o_col + c * 16, w);
          }
        }
      }
      __half2 acc[4] = {__float2half2_rn(0.f), __float2half2_rn(0.f), __float2half2_rn(0.f),
                        __float2half2_rn(0.f)};
      auto weights = [&](auto masked) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = c * 32 + 2 * i;
            float x0 = fmaf(sv[col], sl2, -m_run), x1 = fmaf(sv[col + 1], sl2, -m_run);
            if constexpr (decltype(masked)::value) {
              x0 = (col <= kmax) ? x0 : -INFINITY;
              x1 = (col + 1 <= kmax) ? x1 : -INFINITY;
            }
            // half of the pairs on MUFU (packed fp16 ex2), half on the FMA pipe
            uint32_t e;
            if (i & 1) {
              const float2 y = poly_exp2x2(make_float2(x0, x1));
              e = f2_to_h2(y.x, y.y);
            } else {
              e = ex2_h2(f2_to_h2(x0, x1));
            }
            acc[i & 3] = __hadd2(acc[i & 3], *reinterpret_cast<const __half2*>(&e));
            if constexpr (std::is_same<T, __half>::value) {
              pk[i] = e;
            } else {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&e));
              pk[i] = pack2<__nv_bfloat16>(f.x, f.y);
            }
          }
          tmem_st16(sa + c * 16, pk);                // P_j over the S_j row already read
        }
      };
      if (diag)
        weights(std::true_type());
      else
        weights(std::false_type());
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full + x);
      if (row == 0 && x == 0) PFTRACE(j, 12);
      const float2 s01 = __half22float2(__hadd2(acc[0], acc[1]));
      const float2 s23 = __half22float2(__hadd2(acc[2], acc[3]));
      l_run += (s01.x + s01.y) + (s23.x + s23.y);
    }
    if (ok) ok = __all_sync(0xffffffffu, wait(pv_done + x, (nx - 1) & 1, kDevWaitMma));
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      const bool live = qpos < p.num_tokens;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.out);
      const int64_t base = b * p.o_stride[0] + h * p.o_stride[1] + (int64_t)qpos * p.o_stride[2];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[16];
        tmem_ld16(o_col + c * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] *= inv;
        if (!live) continue;
        if (p.out_dtype == STARKV_F32) {
          float4* d4 = reinterpret_cast<float4*>(dst + 4 * (base + c * 16));
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 2 * (base + c * 16));
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            uint4 w;
            if (p.out_dtype == STARKV_BF16) {
              w.x = pack2<__nv_bfloat16>(v[8 * i], v[8 * i + 1]);
              w.y = pack2<__nv_bfloat16>(v[8 * i + 2], v[8 * i + 3]);
              w.z = pack2<__nv_bfloat16>(v[8 * i + 4], v[8 * i + 5]);
              w.w = pack2<__nv_bfloat16>(v[8 * i + 6], v[8 * i + 7]);
            } else {
              w.x = pack2<__half>(v[8 * i], v[8 * i + 1]);
              w.y = pack2<__half>(v[8 * i + 2], v[8 * i + 3]);
              w.z = pack2<__half>(v[8 * i + 4], v[8 * i + 5]);
              w.w = pack2<__half>(v[8 * i + 6], v[8 * i + 7]);
            }
            d4[i] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace starkv
