// starkv_abi.cu — the extern "C" entry points of libstarkv.so (declared in
// include/starkv.h): validation, launch geometry, workspace carving and the
// kernel launches of the decode step.  No entry point allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "k_logits.cuh"
#include "prefill.cuh"
#include "quant.cuh"
#include "sm100.cuh"
#include "v_latent.cuh"

using namespace starkv;

namespace {

thread_local char g_last_error[256] = "";
// Test hooks (starkv_set_test_hooks): time limit of one device-side wait and a
// K-kernel stage whose copy is never issued.
unsigned long long g_wait_ns = kWaitLimitNs;
int g_skip_unit = -1;
#ifdef STARKV_KTRACE
long long* g_ktrace = nullptr;   // diagnostic builds only
#endif
#ifdef STARKV_PFTRACE
long long* g_pftrace = nullptr;  // diagnostic builds only
#endif

int fail_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return STARKV_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s", cudaGetErrorString(e));
  return STARKV_ERR_LAUNCH;
}

int set_error(int code, const char* msg) {
  snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

constexpr int kMaxDevices = 64;

int device_sm_count(int* dev_out) {
  static int sm_count[kMaxDevices] = {0};
  static int is_sm100[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  if (sm_count[dev] == 0) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return -1;
    is_sm100[dev] = (prop.major == 10 && prop.minor == 0) ? 1 : -1;
    sm_count[dev] = prop.multiProcessorCount;
  }
  if (dev_out) *dev_out = dev;
  return is_sm100[dev] > 0 ? sm_count[dev] : 0;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device).
template <typename K>
int ensure_smem(K kernel, size_t bytes, int slot) {
  constexpr int kSlots = 28;
  static size_t configured[kSlots][kMaxDevices] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || slot < 0 || slot >= kSlots)
    return set_error(STARKV_ERR_INVALID, "internal: kernel attribute slot out of range");
  if (configured[slot][dev] >= bytes) return STARKV_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return fail_launch();
  configured[slot][dev] = bytes;
  return STARKV_OK;
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int max_k_rank(const starkv_layout& l) {
  int m = 0;
  for (int h = 0; h < l.num_kv_heads; ++h) m = l.k_rank[h] > m ? l.k_rank[h] : m;
  return m;
}
int max_v_rank(const starkv_layout& l) {
  int m = 0;
  for (int j = 0; j < l.num_v_blocks; ++j) m = l.v_rank[j] > m ? l.v_rank[j] : m;
  return m;
}
int k_elem_bytes(const starkv_layout& l) { return l.quantized ? 1 : dtype_bytes(l.latent_dtype); }

// K-path geometry: heads per CTA (G) and the shared memory that fits (one CTA
// per SM: it owns all 512 TMEM columns).
struct KGeom {
  int G, rmax, bsum, stage_total;
  size_t smem;
};

KGeom k_geometry(const starkv_layout& l) {
  KGeom g;
  g.rmax = max_k_rank(l);
  const int xb = k_elem_bytes(l);
  const int Hq = l.num_q_heads, qpk = l.num_q_heads / l.num_kv_heads;
  // Largest G whose W matrices leave room for a staging ring of >= 2 tile slots
  // (a tile slot: 128 rows of every distinct KV head of the group).
  for (int G = 4; G >= 1; G >>= 1) {
    if (Hq % G) continue;
    int bsum = 0, tmax = 0;
    for (int grp = 0; grp < Hq / G; ++grp) {
      int s = 0, tb = 0;
      for (int k = 0; k < G; ++k) {
        const int kv = (grp * G + k) / qpk;
        s += l.k_rank[kv];
        if (k == 0 || kv != (grp * G + k - 1) / qpk) tb += 128 * l.k_rank[kv] * xb;
      }
      bsum = s > bsum ? s : bsum;
      tmax = tb > tmax ? tb : tmax;
    }
    const long st = k_stage_total(bsum);
    if (st >= 2L * tmax) {
      g.G = G;
      g.bsum = bsum;
      g.stage_total = (int)st;
      g.smem = (size_t)kKSmemMax;                // one CTA per SM (it owns all 512 TMEM columns)
      return g;
    }
  }
  g.G = 0;
  g.bsum = 0;
  g.smem = 0;
  g.rmax = 0;
  g.stage_total = 0;
  return g;
}

// One split count for every head group: the fewest waves of CTAs times the
// tiles per CTA (plus ~1.5 tiles of fill / prologue per CTA).
int uniform_splits(const starkv_layout& l, int T, int sms) {
  const KGeom g = k_geometry(l);
  if (g.G == 0 || T <= 0) return 1;
  const int ntiles = (T + 127) / 128;
  const long base = (long)l.batch * (l.num_q_heads / g.G);
  const long slots = (long)(sms > 0 ? sms : 148);
  int best = 1;
  double best_t = 1e30;
  for (int ns = 1; ns <= ntiles && ns <= 128; ++ns) {
    const int tiles = (ntiles + ns - 1) / ns;
    const long ctas = base * ns;
    const long waves = (ctas + slots - 1) / slots;
    const double t = (double)waves * (tiles + 1.5);
    if (t < best_t - 1e-9) {
      best_t = t;
      best = ns;
    }
  }
  return best;
}

// Sequence splits of each head group for the K kernel.  The kernel takes a
// split count per head group (so that groups of high ranks could take more
// CTAs); on B200 a cost-balanced choice (the slowest of HBM bytes, tensor
// instructions and drain work per group) measured slower than one uniform
// count (c1: 0.58-0.80 ms against 0.555 ms), so every group gets
// uniform_splits.  override > 0: every group gets that many splits.
struct KSplits {
  int ns_max, S, ngroups;
  int gs[kKMaxGroups];
};

KSplits k_splits(const starkv_layout& l, int T, int sms, int override_ns) {
  KSplits r;
  memset(&r, 0, sizeof(r));
  const KGeom g = k_geometry(l);
  const int G = g.G > 0 ? g.G : 1;
  const int ng = l.num_q_heads / G;
  const int ns = override_ns > 0 ? override_ns : uniform_splits(l, T, sms);
  r.ngroups = ng;
  for (int k = 0; k < ng && k < kKMaxGroups; ++k) r.gs[k] = ns;
  r.ns_max = ns;
  r.S = ns * ng;
  return r;
}

int auto_splits(const starkv_layout& l, int T, int sms) { return k_splits(l, T, sms, 0).ns_max; }

void set_k_splits(KParams& kp, const KSplits& ks) {
  kp.ngroups = ks.ngroups;
  kp.splits_seq = ks.S;
  for (int k = 0; k < kKMaxGroups; ++k) kp.gsplit[k] = ks.gs[k];
}

// Streaming V kernel (int4 latents, all V blocks per CTA): applicability and shared memory.
struct V2Geom {
  bool ok;
  int np, nstages, stage_bytes, b_bytes;
  size_t smem;
};

V2Geom v2_geometry(const starkv_layout& l) {
  V2Geom g;
  memset(&g, 0, sizeof(g));
  if (!l.quantized) return g;
  const int Hq = l.num_q_heads, qpk = Hq / l.num_kv_heads, R = l.v_rank_total;
  if (Hq > kV2MaxHeads) return g;
  (void)qpk;
  // M units are consecutive 128-channel ranges of the whole latent row; every
  // unit's MMA covers all query heads (N = np >= Hq), one shared B tile.
  const int units = (R + 127) / 128;
  g.np = Hq <= 16 ? 16 : 32;
  if (Hq > 32 || units > kV2MaxUnits || units * g.np > 512) return g;
  g.stage_bytes = v2_stage_bytes(R);
  g.b_bytes = g.np * 128;
  const long fixed = (long)kV2Header + (long)kV2Abufs * kV2ABytes + (long)v2_bbufs(R) * g.b_bytes;
  long ns = (227L * 1024 - fixed) / g.stage_bytes;
  if (ns > kV2MaxStages) ns = kV2MaxStages;
  if (ns < 2) return g;
  g.nstages = (int)ns;
  g.smem = v2_smem_bytes(g.nstages, g.stage_bytes, g.b_bytes, v2_bbufs(R));
  if (g.smem < 116 * 1024) g.smem = 116 * 1024;                 // one CTA per SM (512 TMEM columns)
  g.ok = true;
  return g;
}

// V splits of the streaming kernel: one CTA per SM over (split, sequence), at
// least two 64-token tiles per split.
int v2_splits(const starkv_layout& l, int T, int sms) {
  int ns = (sms > 0 ? sms : 148) / l.batch;
  const int cap = (T + 2 * kV2Tile - 1) / (2 * kV2Tile);
  if (ns > cap) ns = cap;
  return ns < 1 ? 1 : ns;
}

// Splits of the V pass: the streaming kernel's own, else the K splits.
int v_splits(const starkv_layout& l, int T, int ns_k, int sms) {
  return v2_geometry(l).ok ? v2_splits(l, T, sms) : ns_k;
}

struct WsLayout {
  size_t err, logits, stats, partial, wimg, weta, total;
};

// stats: K split maxima (B, Hq, ns_k), then V split sums (B, Hq, nsv); partial (B, Hq, nsv, rv_max).
// nsv covers both V kernels (the streaming one may fall back at run time).
WsLayout ws_layout(const starkv_layout& l, int T, int ns_k, int sms) {
  WsLayout w;
  const size_t BH = (size_t)l.batch * l.num_q_heads;
  const int v2 = v_splits(l, T, ns_k, sms);
  const size_t nsv = (size_t)(v2 > ns_k ? v2 : ns_k);
  w.err = 0;
  w.logits = 256;
  w.stats = w.logits + align256(BH * T * sizeof(float));
  w.partial = w.stats + align256(BH * (ns_k + nsv) * sizeof(float));
  w.wimg = w.partial + align256(BH * nsv * max_v_rank(l) * sizeof(float));
  w.weta = w.wimg + align256(BH * (size_t)max_k_rank(l) * 256);
  w.total = w.weta + align256(BH * sizeof(float));
  return w;
}

int validate(const starkv_layout* lp) {
  if (!lp) return set_error(STARKV_ERR_INVALID, "null layout");
  const starkv_layout& l = *lp;
  if (l.abi_version != STARKV_ABI_VERSION) return set_error(STARKV_ERR_INVALID, "layout ABI version mismatch");
  if (l.batch <= 0 || l.num_q_heads <= 0 || l.num_kv_heads <= 0 || l.capacity <= 0)
    return set_error(STARKV_ERR_INVALID, "non-positive batch/heads/capacity");
  if (l.head_dim != STARKV_HEAD_DIM) return set_error(STARKV_ERR_UNSUPPORTED, "head_dim must be 128");
  if (l.num_kv_heads > STARKV_MAX_KV_HEADS || l.num_v_blocks <= 0 || l.num_v_blocks > STARKV_MAX_V_BLOCKS)
    return set_error(STARKV_ERR_UNSUPPORTED, "too many KV heads or V blocks");
  if (l.num_q_heads % l.num_kv_heads) return set_error(STARKV_ERR_INVALID, "num_q_heads % num_kv_heads != 0");
  if (l.latent_dtype < STARKV_F32 || l.latent_dtype > STARKV_BF16)
    return set_error(STARKV_ERR_UNSUPPORTED, "latent dtype");
  const int xb = k_elem_bytes(l);
  int col = 0;
  for (int h = 0; h < l.num_kv_heads; ++h) {
    const int r = l.k_rank[h];
    if (r <= 0 || r % 16 || r > STARKV_MAX_K_RANK)
      return set_error(STARKV_ERR_UNSUPPORTED, "K rank must be a multiple of 16 in [16, 128]");
    if (l.k_col[h] != col) return set_error(STARKV_ERR_INVALID, "k_col is not the prefix sum of k_rank");
    col += r;
    if ((l.k_offset[h] * xb) % 16 || (l.k_batch_stride[h] * xb) % 16 || l.k_offset[h] < 0)
      return set_error(STARKV_ERR_INVALID, "K offsets / batch strides must be 16-byte multiples");
    if (l.k_batch_stride[h] < (int64_t)l.capacity * r)
      return set_error(STARKV_ERR_INVALID, "K batch stride smaller than capacity * rank");
  }
  if (l.k_tiled && l.capacity % 128) return set_error(STARKV_ERR_INVALID, "tiled K layout needs a capacity multiple of 128");
  if (col != l.k_rank_total) return set_error(STARKV_ERR_INVALID, "k_rank_total mismatch");
  const int qpk = l.num_q_heads / l.num_kv_heads;
  int vcol = 0, kv = 0;
  for (int j = 0; j < l.num_v_blocks; ++j) {
    const int r = l.v_rank[j];
    if (r <= 0 || r % 32 || r > kVMaxRank) return set_error(STARKV_ERR_UNSUPPORTED, "V rank must be a multiple of 32 in [32, 1024]");
    if (l.v_col[j] != vcol) return set_error(STARKV_ERR_INVALID, "v_col is not the prefix sum of v_rank");
    if (l.v_first_kv[j] != kv || l.v_num_kv[j] <= 0) return set_error(STARKV_ERR_INVALID, "V blocks must tile the KV heads in order");
    if (l.v_num_kv[j] * qpk > kVMaxHeads) return set_error(STARKV_ERR_UNSUPPORTED, "more than 32 query heads in a V block");
    vcol += r;
    kv += l.v_num_kv[j];
  }
  if (kv != l.num_kv_heads) return set_error(STARKV_ERR_INVALID, "V blocks do not cover the KV heads");
  if (vcol != l.v_rank_total) return set_error(STARKV_ERR_INVALID, "v_rank_total mismatch");
  if (k_geometry(l).G == 0) return set_error(STARKV_ERR_UNSUPPORTED, "K ranks too large for shared memory");
  if (l.num_q_heads / k_geometry(l).G > kKMaxGroups) return set_error(STARKV_ERR_UNSUPPORTED, "more than 64 K head groups");
  return STARKV_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library
// links only the CUDA runtime).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// Tensor map of a strided (B, H, T, 128) 16-bit tensor: boxes of 64 channels x
// 128 tokens of one (head, sequence), 128-byte swizzle, zero fill past T.
int prefill_map(CUtensorMap* map, const void* base, int dtype, int B, int H, int T, const int64_t* strides) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return set_error(STARKV_ERR_LAUNCH, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[4] = {128, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2, (cuuint64_t)strides[0] * 2};
  const cuuint32_t box[4] = {64, 128, 1, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, dtype == STARKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         4, const_cast<void*>(base), dims, gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(STARKV_ERR_INVALID, "cuTensorMapEncodeTiled rejected a prefill tensor");
  return STARKV_OK;
}

int check_device() {
  const int sms = device_sm_count(nullptr);
  if (sms < 0) return set_error(STARKV_ERR_LAUNCH, "no CUDA device");
  if (sms == 0) return set_error(STARKV_ERR_DEVICE, "libstarkv kernels need an sm_100 (B200) device");
  return STARKV_OK;
}

inline unsigned grid1d(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (unsigned)b;
}

template <typename XT, bool QUANT, int G>
int launch_kg(const KParams& kp, const KGeom& g, cudaStream_t st) {
  auto kern = k_logits_kernel<XT, QUANT, G>;
  const int slot = 3 * (QUANT ? 0 : (sizeof(XT) == 4 ? 1 : (std::is_same<XT, __half>::value ? 2 : 3))) + (G == 4 ? 0 : G == 2 ? 1 : 2);
  int rc = ensure_smem(kern, g.smem, slot);
  if (rc) return rc;
  dim3 grid(kp.lay.batch * kp.splits_seq);
  kern<<<grid, kKThreads, g.smem, st>>>(kp);
  return fail_launch();
}

template <typename XT, bool QUANT>
int launch_k(const KParams& kp, const KGeom& g, cudaStream_t st) {
  switch (kp.G) {
    case 4: return launch_kg<XT, QUANT, 4>(kp, g, st);
    case 2: return launch_kg<XT, QUANT, 2>(kp, g, st);
    default: return launch_kg<XT, QUANT, 1>(kp, g, st);
  }
}

int dispatch_k(const KParams& kp, const KGeom& g, cudaStream_t st) {
  if (kp.lay.quantized) return launch_k<int8_t, true>(kp, g, st);
  switch (kp.lay.latent_dtype) {
    case STARKV_F16: return launch_k<__half, false>(kp, g, st);
    case STARKV_BF16: return launch_k<__nv_bfloat16, false>(kp, g, st);
    default: return launch_k<float, false>(kp, g, st);
  }
}

template <typename LT, bool QUANT>
int launch_v(const VParams& vp, int nsplit, cudaStream_t st) {
  auto kern = v_latent_kernel<LT, QUANT>;
  const size_t smem = v_smem_bytes();
  const int slot = 12 + (QUANT ? 0 : (sizeof(LT) == 4 ? 1 : (std::is_same<LT, __half>::value ? 2 : 3)));
  int rc = ensure_smem(kern, smem, slot);
  if (rc) return rc;
  VParams v2 = vp;
  v2.ctiles = (max_v_rank(vp.lay) + kVCtaRank - 1) / kVCtaRank;
  dim3 grid(nsplit, vp.lay.num_v_blocks * v2.ctiles, vp.lay.batch);
  kern<<<grid, kVThreads, smem, st>>>(v2);
  return fail_launch();
}

template <int NP>
int launch_v2(const V2Params& p, const V2Geom& g, cudaStream_t st) {
  auto kern = v_decode_kernel<NP>;
  int rc = ensure_smem(kern, g.smem, NP == 16 ? 16 : 17);
  if (rc) return rc;
  kern<<<dim3(p.nsplit, p.lay.batch), kV2Threads, g.smem, st>>>(p);
  return fail_launch();
}

int dispatch_v(const VParams& vp, int nsplit, cudaStream_t st) {
  if (vp.lay.quantized) return launch_v<uint8_t, true>(vp, nsplit, st);
  switch (vp.lay.latent_dtype) {
    case STARKV_F16: return launch_v<__half, false>(vp, nsplit, st);
    case STARKV_BF16: return launch_v<__nv_bfloat16, false>(vp, nsplit, st);
    default: return launch_v<float, false>(vp, nsplit, st);
  }
}

// Shared front half of decode / logits: validation + K-path parameters.
int prepare_k(const starkv_layout* lay, const starkv_decode_args* a, KParams& kp, KGeom& g) {
  int rc = validate(lay);
  if (rc) return rc;
  if (!a || !a->q || !a->k_u || !a->k_cache || !a->inv_freq) return set_error(STARKV_ERR_INVALID, "null argument");
  if (lay->quantized && !a->k_scales) return set_error(STARKV_ERR_INVALID, "quantised layout needs k_scales");
  if (reinterpret_cast<uintptr_t>(a->k_cache) % 16)
    return set_error(STARKV_ERR_INVALID, "k_cache must be 16-byte aligned");
  if (a->num_tokens <= 0 || a->num_tokens > lay->capacity)
    return set_error(STARKV_ERR_INVALID, "num_tokens outside (0, capacity]");
  rc = check_device();
  if (rc) return rc;
  g = k_geometry(*lay);
  memset(&kp, 0, sizeof(kp));
  kp.lay = *lay;
  kp.q = a->q;
  kp.k_u = a->k_u;
  kp.k_cache = a->k_cache;
  kp.k_scales = reinterpret_cast<const __half*>(a->k_scales);
  kp.q_dtype = a->q_dtype;
  kp.w_dtype = a->w_dtype;
  kp.T = a->num_tokens;
  kp.G = g.G;
  kp.rmax = g.rmax;
  kp.bsum = g.bsum;
  kp.stage_total = g.stage_total;
  kp.inv_freq = a->inv_freq;
  kp.wait_ns = g_wait_ns;
  kp.skip_unit = g_skip_unit;
#ifdef STARKV_KTRACE
  kp.trace = g_ktrace;
#endif
  return STARKV_OK;
}

template <typename LT, bool QUANT>
int launch_pa(const starkv_layout& l, const void* hidden, int H, const void* vs_k, const void* vs_v, int slot,
              void* k_cache, const void* k_scales, void* v_cache, void* v_params, void* k_out, void* v_out,
              cudaStream_t st) {
  auto kern = project_append_kernel<LT, QUANT>;
  const size_t smem = (size_t)kPaSeqOf<LT>() * H * sizeof(LT);
  const int slotid = 18 + 2 * (sizeof(LT) == 4 ? 0 : std::is_same<LT, __half>::value ? 1 : 2) + (QUANT ? 1 : 0);
  int rc = ensure_smem(kern, smem, slotid > 23 ? 23 : slotid);
  if (rc) return rc;
  const int nchunks = (l.k_rank_total + 31) / 32 + l.v_rank_total / 32;
  kern<<<dim3(nchunks, (l.batch + kPaSeqOf<LT>() - 1) / kPaSeqOf<LT>()), kPaWarps * 32, smem, st>>>(
      l, (const LT*)hidden, H, (const LT*)vs_k, (const LT*)vs_v, slot, k_cache, (const __half*)k_scales, v_cache,
      (__half2*)v_params, (LT*)k_out, (LT*)v_out);
  return fail_launch();
}

}  // namespace

extern "C" {

size_t starkv_layout_size(void) { return sizeof(starkv_layout); }

int starkv_validate_layout(const starkv_layout* lay) { return validate(lay); }

const char* starkv_last_error(void) { return g_last_error; }

int32_t starkv_auto_splits(const starkv_layout* lay, int32_t num_tokens) {
  if (validate(lay)) return 1;
  const int sms = device_sm_count(nullptr);
  return auto_splits(*lay, num_tokens, sms > 0 ? sms : 148);
}

int starkv_project_append(const starkv_layout* lay, const void* hidden, int32_t hidden_size, const void* vs_k,
                          const void* vs_v, int32_t slot, void* k_cache, const void* k_scales, void* v_cache,
                          void* v_params, void* k_lat_out, void* v_lat_out, starkv_stream_t stream) {
  int rc = validate(lay);
  if (rc) return rc;
  const starkv_layout& l = *lay;
  const int eb = dtype_bytes(l.latent_dtype);
  if (!hidden || !vs_k || !vs_v || !k_cache || !v_cache || slot < 0 || slot >= l.capacity || hidden_size <= 0)
    return set_error(STARKV_ERR_INVALID, "bad arguments (slot beyond capacity?)");
  if (l.quantized && (!k_scales || !v_params)) return set_error(STARKV_ERR_INVALID, "null scales");
  if ((hidden_size * eb) % 16 || (reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(vs_k) |
                                  reinterpret_cast<uintptr_t>(vs_v)) % 16)
    return set_error(STARKV_ERR_INVALID, "hidden rows and VS matrices must be 16-byte aligned");
  if ((size_t)8 * hidden_size * eb > (size_t)kKSmemMax - 32 * 1024)
    return set_error(STARKV_ERR_UNSUPPORTED, "hidden size too large for the fused projection");
  rc = check_device();
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  switch (l.latent_dtype) {
    case STARKV_F16:
      return l.quantized ? launch_pa<__half, true>(l, hidden, hidden_size, vs_k, vs_v, slot, k_cache, k_scales, v_cache, v_params, k_lat_out, v_lat_out, st)
                         : launch_pa<__half, false>(l, hidden, hidden_size, vs_k, vs_v, slot, k_cache, k_scales, v_cache, v_params, k_lat_out, v_lat_out, st);
    case STARKV_BF16:
      return l.quantized ? launch_pa<__nv_bfloat16, true>(l, hidden, hidden_size, vs_k, vs_v, slot, k_cache, k_scales, v_cache, v_params, k_lat_out, v_lat_out, st)
                         : launch_pa<__nv_bfloat16, false>(l, hidden, hidden_size, vs_k, vs_v, slot, k_cache, k_scales, v_cache, v_params, k_lat_out, v_lat_out, st);
    default:
      return l.quantized ? launch_pa<float, true>(l, hidden, hidden_size, vs_k, vs_v, slot, k_cache, k_scales, v_cache, v_params, k_lat_out, v_lat_out, st)
                         : launch_pa<float, false>(l, hidden, hidden_size, vs_k, vs_v, slot, k_cache, k_scales, v_cache, v_params, k_lat_out, v_lat_out, st);
  }
}

int starkv_decode_workspace_size(const starkv_layout* lay, int32_t num_tokens, int32_t num_splits, size_t* bytes) {
  int rc = validate(lay);
  if (rc) return rc;
  if (!bytes || num_tokens <= 0) return set_error(STARKV_ERR_INVALID, "bad arguments");
  const int ns = num_splits > 0 ? num_splits : starkv_auto_splits(lay, num_tokens);
  const int sms = device_sm_count(nullptr);
  *bytes = ws_layout(*lay, num_tokens, ns, sms > 0 ? sms : 148).total;
  return STARKV_OK;
}

int starkv_quantize_prefill(const starkv_layout* lay, const void* k_lat, const void* v_lat, int32_t num_tokens,
                            void* k_cache, void* k_scales, void* v_cache, void* v_params, starkv_stream_t stream) {
  int rc = validate(lay);
  if (rc) return rc;
  if (!k_lat || !v_lat || !k_cache || !v_cache || num_tokens < 0 || num_tokens > lay->capacity)
    return set_error(STARKV_ERR_INVALID, "bad arguments");
  if (lay->quantized && (!k_scales || !v_params)) return set_error(STARKV_ERR_INVALID, "null scales");
  rc = check_device();
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const starkv_layout& l = *lay;
  if (!l.quantized) return starkv_append(lay, k_lat, v_lat, num_tokens, 0, k_cache, k_scales, v_cache, v_params, stream);
  // spread the prompt's tokens over about two waves of CTAs (at least 256 tokens each)
  const int kz = std::max(1, std::min((num_tokens + 255) / 256,
                                      (2 * 148 + l.num_kv_heads * l.batch - 1) / (l.num_kv_heads * l.batch)));
  dim3 kg(l.num_kv_heads, l.batch, kz);
  switch (l.latent_dtype) {
    case STARKV_F16:
      k_prefill_quant_kernel<__half><<<kg, 256, 0, st>>>(l, (const __half*)k_lat, num_tokens, (int8_t*)k_cache, (__half*)k_scales);
      break;
    case STARKV_BF16:
      k_prefill_quant_kernel<__nv_bfloat16><<<kg, 256, 0, st>>>(l, (const __nv_bfloat16*)k_lat, num_tokens, (int8_t*)k_cache, (__half*)k_scales);
      break;
    default:
      k_prefill_quant_kernel<float><<<kg, 256, 0, st>>>(l, (const float*)k_lat, num_tokens, (int8_t*)k_cache, (__half*)k_scales);
  }
  rc = fail_launch();
  if (rc || num_tokens == 0) return rc;
  const int64_t nthreads = (int64_t)l.batch * num_tokens * (l.v_rank_total / 32) * 32;
  const unsigned grid = grid1d(nthreads, 256);
  switch (l.latent_dtype) {
    case STARKV_F16:
      v_quant_kernel<__half><<<grid, 256, 0, st>>>(l, (const __half*)v_lat, num_tokens, 0, (uint8_t*)v_cache, (__half2*)v_params);
      break;
    case STARKV_BF16:
      v_quant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(l, (const __nv_bfloat16*)v_lat, num_tokens, 0, (uint8_t*)v_cache, (__half2*)v_params);
      break;
    default:
      v_quant_kernel<float><<<grid, 256, 0, st>>>(l, (const float*)v_lat, num_tokens, 0, (uint8_t*)v_cache, (__half2*)v_params);
  }
  return fail_launch();
}

int starkv_append(const starkv_layout* lay, const void* k_lat, const void* v_lat, int32_t num_tokens,
                  int32_t start_slot, void* k_cache, const void* k_scales, void* v_cache, void* v_params,
                  starkv_stream_t stream) {
  int rc = validate(lay);
  if (rc) return rc;
  if (!k_lat || !v_lat || !k_cache || !v_cache || num_tokens < 0 || start_slot < 0 ||
      (int64_t)start_slot + num_tokens > lay->capacity)
    return set_error(STARKV_ERR_INVALID, "bad arguments (slots beyond capacity?)");
  if (lay->quantized && (!k_scales || !v_params)) return set_error(STARKV_ERR_INVALID, "null scales");
  rc = check_device();
  if (rc) return rc;
  if (num_tokens == 0) return STARKV_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const starkv_layout& l = *lay;
  if (!l.quantized) {
    const int64_t n = (int64_t)l.batch * num_tokens * (l.k_rank_total + l.v_rank_total);
    const unsigned grid = grid1d(n, 256);
    switch (l.latent_dtype) {
      case STARKV_F16:
        copy_append_kernel<__half><<<grid, 256, 0, st>>>(l, (const __half*)k_lat, (const __half*)v_lat, num_tokens, start_slot, (__half*)k_cache, (__half*)v_cache);
        break;
      case STARKV_BF16:
        copy_append_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(l, (const __nv_bfloat16*)k_lat, (const __nv_bfloat16*)v_lat, num_tokens, start_slot, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache);
        break;
      default:
        copy_append_kernel<float><<<grid, 256, 0, st>>>(l, (const float*)k_lat, (const float*)v_lat, num_tokens, start_slot, (float*)k_cache, (float*)v_cache);
    }
    return fail_launch();
  }
  const int64_t nk = (int64_t)l.batch * num_tokens * l.k_rank_total;
  const int64_t nv = (int64_t)l.batch * num_tokens * (l.v_rank_total / 32) * 32;
  switch (l.latent_dtype) {
    case STARKV_F16:
      k_append_quant_kernel<__half><<<grid1d(nk, 256), 256, 0, st>>>(l, (const __half*)k_lat, num_tokens, start_slot, (int8_t*)k_cache, (const __half*)k_scales);
      v_quant_kernel<__half><<<grid1d(nv, 256), 256, 0, st>>>(l, (const __half*)v_lat, num_tokens, start_slot, (uint8_t*)v_cache, (__half2*)v_params);
      break;
    case STARKV_BF16:
      k_append_quant_kernel<__nv_bfloat16><<<grid1d(nk, 256), 256, 0, st>>>(l, (const __nv_bfloat16*)k_lat, num_tokens, start_slot, (int8_t*)k_cache, (const __half*)k_scales);
      v_quant_kernel<__nv_bfloat16><<<grid1d(nv, 256), 256, 0, st>>>(l, (const __nv_bfloat16*)v_lat, num_tokens, start_slot, (uint8_t*)v_cache, (__half2*)v_params);
      break;
    default:
      k_append_quant_kernel<float><<<grid1d(nk, 256), 256, 0, st>>>(l, (const float*)k_lat, num_tokens, start_slot, (int8_t*)k_cache, (const __half*)k_scales);
      v_quant_kernel<float><<<grid1d(nv, 256), 256, 0, st>>>(l, (const float*)v_lat, num_tokens, start_slot, (uint8_t*)v_cache, (__half2*)v_params);
  }
  return fail_launch();
}

int starkv_decode_attention(const starkv_layout* lay, const starkv_decode_args* a, starkv_stream_t stream) {
  KParams kp;
  KGeom g;
  int rc = prepare_k(lay, a, kp, g);
  if (rc) return rc;
  if (!a->v_cache || !a->v_u || !a->out || !a->workspace) return set_error(STARKV_ERR_INVALID, "null argument");
  if (lay->quantized && !a->v_params) return set_error(STARKV_ERR_INVALID, "quantised layout needs v_params");
  if (reinterpret_cast<uintptr_t>(a->workspace) % 256) return set_error(STARKV_ERR_INVALID, "workspace not 256-byte aligned");
  const int T = a->num_tokens;
  const int sms = device_sm_count(nullptr);
  const KSplits ks = k_splits(*lay, T, sms, a->num_splits);
  const int ns = ks.ns_max;
  const WsLayout w = ws_layout(*lay, T, ns, sms);
  if (a->workspace_bytes < w.total) return set_error(STARKV_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  set_k_splits(kp, ks);

  const int ntiles = (T + 127) / 128;
  const int tiles_per = (ntiles + ns - 1) / ns;
  kp.mask = a->mask;
  kp.logits = reinterpret_cast<float*>(ws + w.logits);
  // W of every (sequence, query head) once, ahead of the K kernel (its CTAs bulk-copy theirs)
  kp.wstride = max_k_rank(*lay) * 256;
  kp.wpre = ws + w.wimg;
  kp.weta = reinterpret_cast<float*>(ws + w.weta);
  kp.smax = reinterpret_cast<float*>(ws + w.stats);     // split maxima, then split sums (same region)
  kp.err = reinterpret_cast<int*>(ws + w.err);
  kp.nsplit = ns;
  kp.tps = tiles_per * 128;
  const float log2e = 1.4426950408889634f;
  kp.out_scale = a->scaling * log2e;
  kp.mask_scale = log2e;
  cudaEvent_t const* ev = reinterpret_cast<cudaEvent_t const*>(a->events);
  if (ev) cudaEventRecord(ev[0], st);
  {
    const dim3 wg(lay->num_q_heads, lay->batch);
    if (lay->quantized)
      k_wprep_kernel<true><<<wg, 256, 0, st>>>(kp, ws + w.wimg, reinterpret_cast<float*>(ws + w.weta));
    else
      k_wprep_kernel<false><<<wg, 256, 0, st>>>(kp, ws + w.wimg, reinterpret_cast<float*>(ws + w.weta));
    rc = fail_launch();
    if (rc) return rc;
  }
  rc = dispatch_k(kp, g, st);
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[1], st);

  if (lay->quantized &&
      (reinterpret_cast<uintptr_t>(a->v_cache) % 16 || reinterpret_cast<uintptr_t>(a->v_params) % 16))
    return set_error(STARKV_ERR_INVALID, "v_cache and v_params must be 16-byte aligned");
  const V2Geom vg = v2_geometry(*lay);
  const bool stream_v = vg.ok;
  const int nsv = stream_v ? v2_splits(*lay, T, sms) : ns;
  float* lsum = kp.smax + (size_t)lay->batch * lay->num_q_heads * ns;
  float* partial = reinterpret_cast<float*>(ws + w.partial);
  if (stream_v) {
    V2Params v2;
    memset(&v2, 0, sizeof(v2));
    v2.lay = *lay;
    v2.logits = kp.logits;
    v2.smax = kp.smax;
    v2.lsum = lsum;
    v2.v_cache = reinterpret_cast<const uint8_t*>(a->v_cache);
    v2.v_params = reinterpret_cast<const uint8_t*>(a->v_params);
    v2.partial = partial;
    v2.err = kp.err;
    v2.T = T;
    v2.nsplit = nsv;
    v2.nsplit_k = ns;
    v2.tps = ((T + nsv * kV2Tile - 1) / (nsv * kV2Tile)) * kV2Tile;
    v2.rv_max = max_v_rank(*lay);
    v2.nstages = vg.nstages;
    v2.stage_bytes = vg.stage_bytes;
    v2.b_bytes = vg.b_bytes;
    rc = vg.np == 16 ? launch_v2<16>(v2, vg, st) : launch_v2<32>(v2, vg, st);
  } else {
    VParams vp;
    memset(&vp, 0, sizeof(vp));
    vp.lay = *lay;
    vp.logits = kp.logits;
    vp.smax = kp.smax;
    vp.lsum = lsum;
    vp.v_cache = a->v_cache;
    vp.v_params = reinterpret_cast<const __half2*>(a->v_params);
    vp.partial = partial;
    vp.T = T;
    vp.nsplit = ns;
    vp.nsplit_k = ns;
    vp.tps = kp.tps;
    vp.rv_max = max_v_rank(*lay);
    vp.err = kp.err;
    rc = dispatch_v(vp, ns, st);
  }
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[2], st);

  CombineParams cp;
  memset(&cp, 0, sizeof(cp));
  cp.lay = *lay;
  cp.partial = partial;
  cp.lsum = lsum;
  cp.v_u = a->v_u;
  cp.out = a->out;
  cp.w_dtype = a->w_dtype;
  cp.out_dtype = a->out_dtype;
  cp.nsplit = nsv;
  cp.rv_max = max_v_rank(*lay);
  combine_kernel<<<dim3(lay->num_q_heads, lay->batch), 128, 0, st>>>(cp);
  rc = fail_launch();
  if (!rc && ev) cudaEventRecord(ev[3], st);
  return rc;
}

int starkv_k_logits(const starkv_layout* lay, const starkv_decode_args* a, float* logits, starkv_stream_t stream) {
  KParams kp;
  KGeom g;
  int rc = prepare_k(lay, a, kp, g);
  if (rc) return rc;
  if (!logits) return set_error(STARKV_ERR_INVALID, "logits is required");
  const int T = a->num_tokens;
  const KSplits ks = k_splits(*lay, T, device_sm_count(nullptr), a->num_splits);
  const int ns = ks.ns_max;
  const int ntiles = (T + 127) / 128;
  set_k_splits(kp, ks);
  kp.logits = logits;
  kp.nsplit = ns;
  kp.tps = ((ntiles + ns - 1) / ns) * 128;
  kp.out_scale = 1.0f;
  kp.mask_scale = 1.0f;
  return dispatch_k(kp, g, (cudaStream_t)stream);
}

int starkv_v_latent(const starkv_layout* lay, const float* probs, int32_t num_tokens, const void* v_cache,
                    const void* v_params, float* out, starkv_stream_t stream) {
  int rc = validate(lay);
  if (rc) return rc;
  if (!probs || !v_cache || !out || num_tokens <= 0 || num_tokens > lay->capacity ||
      (lay->quantized && !v_params))
    return set_error(STARKV_ERR_INVALID, "bad arguments");
  rc = check_device();
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t n = (size_t)lay->batch * lay->num_q_heads * lay->v_rank_total * sizeof(float);
  if (cudaMemsetAsync(out, 0, n, st) != cudaSuccess) return fail_launch();
  VParams vp;
  memset(&vp, 0, sizeof(vp));
  vp.lay = *lay;
  vp.probs = probs;
  vp.v_cache = v_cache;
  vp.v_params = reinterpret_cast<const __half2*>(v_params);
  vp.partial = out;
  vp.T = num_tokens;
  vp.nsplit = 1;
  vp.nsplit_k = 1;
  vp.tps = num_tokens;
  vp.rv_max = max_v_rank(*lay);
  return dispatch_v(vp, 1, st);
}

int starkv_quantize_split(const void* x, int32_t dtype, int64_t rows, int32_t r, int32_t split_r, void* up_q,
                          void* s_up, void* lo_q, void* s_lo, starkv_stream_t stream) {
  if (!x || rows < 0 || r <= 0 || split_r < 0 || split_r > r || dtype < STARKV_F32 || dtype > STARKV_BF16)
    return set_error(STARKV_ERR_INVALID, "bad arguments");
  if ((split_r > 0 && (!up_q || !s_up)) || (split_r < r && (!lo_q || !s_lo)))
    return set_error(STARKV_ERR_INVALID, "null output");
  int rc = check_device();
  if (rc) return rc;
  if (rows == 0) return STARKV_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = grid1d(rows * 32, 256);
  switch (dtype) {
    case STARKV_F16:
      split_quant_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, rows, r, split_r, (int8_t*)up_q, (__half*)s_up, (uint8_t*)lo_q, (__half*)s_lo);
      break;
    case STARKV_BF16:
      split_quant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, rows, r, split_r, (int8_t*)up_q, (__half*)s_up, (uint8_t*)lo_q, (__half*)s_lo);
      break;
    default:
      split_quant_kernel<float><<<grid, 256, 0, st>>>((const float*)x, rows, r, split_r, (int8_t*)up_q, (__half*)s_up, (uint8_t*)lo_q, (__half*)s_lo);
  }
  return fail_launch();
}

#ifdef STARKV_KTRACE
// Diagnostic builds only: K kernel timeline buffer (16 x 1024 job stamps of CTA 0,
// then start / end of CTAs 0..1023), or null to stop.
extern "C" int starkv_debug_ktrace(void* buf) {
  g_ktrace = reinterpret_cast<long long*>(buf);
  return STARKV_OK;
}
#endif

#ifdef STARKV_PFTRACE
// Diagnostic builds only: prefill kernel timeline of CTA 0 (16 stamps per key
// tile, 512 tiles at most), or null to stop.
extern "C" int starkv_debug_pftrace(void* buf) {
  g_pftrace = reinterpret_cast<long long*>(buf);
  return STARKV_OK;
}
#endif

int starkv_set_test_hooks(int64_t wait_limit_ns, int32_t skip_copy_unit) {
  g_wait_ns = wait_limit_ns > 0 ? (unsigned long long)wait_limit_ns : kWaitLimitNs;
  g_skip_unit = skip_copy_unit;
  return STARKV_OK;
}

int starkv_read_device_error(void* workspace, int* out_code, starkv_stream_t stream) {
  if (!workspace || !out_code) return set_error(STARKV_ERR_INVALID, "bad arguments");
  cudaStream_t st = (cudaStream_t)stream;
  int code = 0;
  if (cudaMemcpyAsync(&code, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return fail_launch();
  if (cudaStreamSynchronize(st) != cudaSuccess) return fail_launch();
  *out_code = code;
  if (code && cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return fail_launch();
  return STARKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode attention without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they run a
// decode step: code running inside another framework's memory pool, plugin
// hosts that hand over only input and output buffers, or processes whose
// allocator is locked down.  For them the scratch of the decode step lives in
// this fixed, file-scope device array.  Every GPU that loads the library
// reserves it until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = 32u << 20;  // 32 MiB
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch, looked up once per device (with that
// device current) on the first call made on it.
uint8_t* static_scratch_ptr(int* rc) {
  static void* ptr[kMaxDevices] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *rc = set_error(STARKV_ERR_LAUNCH, "no current CUDA device");
    return nullptr;
  }
  if (!ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) {
      *rc = fail_launch();
      if (!*rc) *rc = set_error(STARKV_ERR_LAUNCH, "cudaGetSymbolAddress(g_static_scratch) failed");
      return nullptr;
    }
    ptr[dev] = p;
  }
  *rc = STARKV_OK;
  return reinterpret_cast<uint8_t*>(ptr[dev]);
}

}  // namespace

extern "C" {

size_t starkv_static_scratch_bytes(void) { return kStaticScratchBytes; }

int starkv_static_read_device_error(int* out_code, starkv_stream_t stream) {
  if (!out_code) return set_error(STARKV_ERR_INVALID, "null out_code");
  int rc = STARKV_OK;
  uint8_t* scratch = static_scratch_ptr(&rc);
  if (rc) return rc;
  return starkv_read_device_error(scratch, out_code, stream);
}

int starkv_decode_attention_static(const starkv_layout* lay, const starkv_decode_args* args,
                                   starkv_stream_t stream) {
  int rc = validate(lay);
  if (rc) return rc;
  if (!args) return set_error(STARKV_ERR_INVALID, "null argument");
  if (args->num_tokens <= 0 || args->num_tokens > lay->capacity)
    return set_error(STARKV_ERR_INVALID, "num_tokens outside (0, capacity]");
  const int sms = device_sm_count(nullptr);
  if (sms < 0) return set_error(STARKV_ERR_LAUNCH, "no CUDA device");
  const int ns = args->num_splits > 0 ? args->num_splits : auto_splits(*lay, args->num_tokens, sms);
  const size_t need = ws_layout(*lay, args->num_tokens, ns, sms).total;
  if (need > kStaticScratchBytes) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "decode step needs %zu bytes of scratch, above the %zu-byte static scratch of "
             "starkv_decode_attention_static; use starkv_decode_attention with a workspace",
             need, kStaticScratchBytes);
    return set_error(STARKV_ERR_WORKSPACE, msg);
  }
  uint8_t* scratch = static_scratch_ptr(&rc);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // The array keeps whatever the previous call left: the error word must start at zero.
  if (cudaMemsetAsync(scratch, 0, 256, st) != cudaSuccess) return fail_launch();
  starkv_decode_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kStaticScratchBytes;
  return starkv_decode_attention(lay, &a, stream);
}

int starkv_prefill_attention(const starkv_prefill_args* a, starkv_stream_t stream) {
  if (!a || !a->q || !a->k || !a->v || !a->out) return set_error(STARKV_ERR_INVALID, "null argument");
  if (a->dtype != STARKV_F16 && a->dtype != STARKV_BF16)
    return set_error(STARKV_ERR_UNSUPPORTED, "prefill attention takes fp16 or bf16 q / k / v");
  if (a->out_dtype != STARKV_F16 && a->out_dtype != STARKV_BF16 && a->out_dtype != STARKV_F32)
    return set_error(STARKV_ERR_INVALID, "bad out_dtype");
  if (a->batch <= 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->num_tokens <= 0 ||
      a->num_q_heads % a->num_kv_heads != 0)
    return set_error(STARKV_ERR_INVALID, "bad batch / head / token counts");
  const int64_t* strides[3] = {a->q_strides, a->k_strides, a->v_strides};
  const void* ptrs[3] = {a->q, a->k, a->v};
  for (int i = 0; i < 3; ++i) {
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16 != 0)
      return set_error(STARKV_ERR_INVALID, "q / k / v must be 16-byte aligned");
    for (int d = 0; d < 3; ++d)
      if (strides[i][d] % 8 != 0 || strides[i][d] < 0)
        return set_error(STARKV_ERR_INVALID, "q / k / v strides must be non-negative multiples of 8 elements");
  }
  const int oe = a->out_dtype == STARKV_F32 ? 4 : 8;
  if (reinterpret_cast<uintptr_t>(a->out) % 16 != 0)
    return set_error(STARKV_ERR_INVALID, "out must be 16-byte aligned");
  for (int d = 0; d < 3; ++d)
    if (a->out_strides[d] % oe != 0 || a->out_strides[d] < 0)
      return set_error(STARKV_ERR_INVALID, "out strides must be non-negative multiples of 16 bytes");
  int rc = check_device();
  if (rc) return rc;
  PrefillParams p;
  memset(&p, 0, sizeof(p));
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.out = a->out;
  for (int d = 0; d < 3; ++d) {
    p.q_stride[d] = a->q_strides[d];
    p.k_stride[d] = a->k_strides[d];
    p.v_stride[d] = a->v_strides[d];
    p.o_stride[d] = a->out_strides[d];
  }
  p.batch = a->batch;
  p.num_q_heads = a->num_q_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.num_tokens = a->num_tokens;
  p.n_qtiles = (a->num_tokens + kPfTile - 1) / kPfTile;
  p.out_dtype = a->out_dtype;
  p.scale_log2 = a->scaling * 1.4426950408889634f;
  p.err = a->error_word;
  p.wait_ns = g_wait_ns;
#ifdef STARKV_PFTRACE
  p.trace = g_pftrace;
#endif
  // V operand descriptor (MN-major, 128-byte swizzle): the second 64-channel box
  // sits 16 KB along N, 8-token groups 1 KB apart along K
  p.v_lbo = 16384;
  p.v_sbo = 1024;
  CUtensorMap tq, tk, tv;
  if ((rc = prefill_map(&tq, a->q, a->dtype, a->batch, a->num_q_heads, a->num_tokens, a->q_strides)) ||
      (rc = prefill_map(&tk, a->k, a->dtype, a->batch, a->num_kv_heads, a->num_tokens, a->k_strides)) ||
      (rc = prefill_map(&tv, a->v, a->dtype, a->batch, a->num_kv_heads, a->num_tokens, a->v_strides)))
    return rc;
  const int64_t ctas = (int64_t)((p.n_qtiles + 1) / 2) * a->num_q_heads * a->batch;
  if (ctas > 0x7fffffff) return set_error(STARKV_ERR_UNSUPPORTED, "too many query tiles");
  cudaStream_t st = (cudaStream_t)stream;
  if (a->dtype == STARKV_F16) {
    rc = ensure_smem(prefill_attn2_kernel<__half>, kPf2Smem, 24);
    if (rc) return rc;
    prefill_attn2_kernel<__half><<<(unsigned)ctas, kPf2Threads, kPf2Smem, st>>>(p, tq, tk, tv);
  } else {
    rc = ensure_smem(prefill_attn2_kernel<__nv_bfloat16>, kPf2Smem, 25);
    if (rc) return rc;
    prefill_attn2_kernel<__nv_bfloat16><<<(unsigned)ctas, kPf2Threads, kPf2Smem, st>>>(p, tq, tk, tv);
  }
  return fail_launch();
}

}  // extern "C"
