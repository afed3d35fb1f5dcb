// int8 weight-only GEMV / skinny GEMM for the HeartMuLa decode path (sm_100a).
//
// Replaces the reference's `_gemv8` Triton kernel and its `int8_mm` dispatcher
// (app/kernels.py:20-54) and fuses what surrounds it in Stack.decode
// (app/engine.py:180-211): RMSNorm or an int8 embedding gather in the
// prologue; residual add, RoPE + KV-cache write, or SiLU*mul in the epilogue.
//
// Design (HBM-bound: every weight byte is read exactly once per frame):
//  * CTA tile = 64 weight rows x `kspan` columns (kspan <= 1024, split-K over
//    the grid's y dimension).  One thread issues TMA tile loads for the whole
//    tile at CTA start, before griddepcontrol.wait, so weight streaming of
//    this launch overlaps the tail of the previous one.  Tiles land 128B-
//    swizzled so the fragment reads below are bank-conflict free.
//  * Tensor-core MMA m16n8k16 with the weights as the 16-row A operand and up
//    to 8*MT activation rows as the n dimension ("swap AB"): at R = 8 rows the
//    MMA n = 8 carries no padding.  The int8 -> fp16 conversion is exact, the
//    accumulation is fp32, and the per-row scale is applied afterwards in fp32,
//    exactly where _gemv8 applies it.
//  * K inside a 128-column block is permuted consistently for A and B so every
//    lane reads 32 contiguous weight bytes and 64 contiguous activation bytes.
//  * Split-K partials go to a scratch buffer; the last CTA of a tile (atomic
//    ticket) sums them in split order (deterministic) and runs the epilogue,
//    then re-arms the ticket to zero.
#include <cudaTypedefs.h>

#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "hm_common.cuh"

namespace {

constexpr int kRows = 64;     // weight rows per CTA tile
constexpr int kBlkK = 128;    // k columns (bytes) per TMA box / mbarrier
constexpr int kBoxRows = 32;  // rows per TMA box (two boxes per block)
constexpr int kThreads = 128;
constexpr int kMaxKspan = 1024;
constexpr int kMaxBlocks = kMaxKspan / kBlkK;
constexpr int kMaxM = 32;

struct GemvParams {
  hm_gemv_desc d;
  int kspan, nsplit, ntiles;
};

struct SmemLayout {
  int w_off, x_off, acc_off, sq_off, scale_off, inv_off, flag_off, bar_off, total;
  int xp;  // x row pitch in bytes
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int kspan, int mrows) {
  SmemLayout L;
  const int nblk = kspan / kBlkK;
  L.w_off = 0;
  L.xp = kspan * 2 + 16;
  L.x_off = nblk * kBlkK * kRows;                      // multiple of 8192 -> 1024-aligned
  L.acc_off = align_up(L.x_off + mrows * L.xp, 16);
  L.sq_off = L.acc_off + kRows * (mrows + 1) * 4;
  L.scale_off = L.sq_off + kRows * mrows * 4;
  L.inv_off = L.scale_off + kRows * 4;
  L.flag_off = L.inv_off + kMaxM * 4;
  L.bar_off = align_up(L.flag_off + 16, 8);
  L.total = L.bar_off + kMaxBlocks * 8;
  return L;
}

// Swizzled position of 16-byte chunk c inside an activation row (bank-conflict
// free for the B-fragment reads: lanes t and t+2 land in different banks).
__device__ __forceinline__ int xchunk(int c) { return c ^ (((c >> 3) & 1) << 1); }

struct RowRef {
  const hm_row_src* s;
  int row;
};

__device__ __forceinline__ RowRef row_of(const hm_gemv_desc& d, int m) {
  const int sel = d.interleave ? (m & 1) : 0;
  const int local = d.interleave ? (m >> 1) : m;
  RowRef r;
  r.s = &d.src[sel];
  r.row = local * r.s->row_mul + r.s->row_add;
  return r;
}

// 8 consecutive activations of row m starting at column k, after the prologue transform.
__device__ __forceinline__ uint4 load_x8(const hm_gemv_desc& d, int m, int k, float inv, int* err) {
  if (k >= d.K) return make_uint4(0, 0, 0, 0);  // column tail of a K that is not a multiple of 128
  const RowRef rr = row_of(d, m);
  const hm_row_src& s = *rr.s;
  if (s.mode == HM_SRC_EMB) {
    int64_t id = s.tok[(int64_t)rr.row * s.tok_ld + s.tok_col] + s.tok_off;
    if (id < 0 || id >= s.erows) {
      report_error(err, HM_ERR_BADINDEX);
      return make_uint4(0, 0, 0, 0);
    }
    const uint2 q = *reinterpret_cast<const uint2*>(s.etab + id * (int64_t)d.K + k);
    const float sc = __half2float(reinterpret_cast<const __half*>(s.escale)[id]);
    const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
    uint4 out;
    __half* oh = reinterpret_cast<__half*>(&out);
#pragma unroll
    for (int j = 0; j < 8; ++j) oh[j] = __float2half_rn(static_cast<float>(qb[j]) * sc);
    return out;
  }
  const __half* xr = reinterpret_cast<const __half*>(s.x) + (int64_t)rr.row * s.ldx + k;
  uint4 v = *reinterpret_cast<const uint4*>(xr);
  if (s.mode == HM_SRC_RMS) {
    const __half* g = reinterpret_cast<const __half*>(s.gamma) + k;
    const uint4 gv = *reinterpret_cast<const uint4*>(g);
    __half* vh = reinterpret_cast<__half*>(&v);
    const __half* gh = reinterpret_cast<const __half*>(&gv);
#pragma unroll
    for (int j = 0; j < 8; ++j) vh[j] = hmul_rn(__float2half_rn(__half2float(vh[j]) * inv), gh[j]);
  }
  return v;
}

template <int MT, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_i8_kernel(const __grid_constant__ CUtensorMap wmap,
                                                           const __grid_constant__ GemvParams P) {
  constexpr int MROWS = 8 * MT;
  constexpr int MP = MROWS + 1;
  extern __shared__ __align__(1024) uint8_t smem[];
  const hm_gemv_desc& d = P.d;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int kspan = P.kspan, nblk = kspan / kBlkK;
  const int k0 = split * kspan;
  const int M = d.M;
  const SmemLayout L = smem_layout(kspan, MROWS);
  uint8_t* wsm = smem + L.w_off;
  uint8_t* xsm = smem + L.x_off;
  float* acc_s = reinterpret_cast<float*>(smem + L.acc_off);
  float* sq_s = reinterpret_cast<float*>(smem + L.sq_off);
  float* scale_s = reinterpret_cast<float*>(smem + L.scale_off);
  float* inv_s = reinterpret_cast<float*>(smem + L.inv_off);
  int* flag_s = reinterpret_cast<int*>(smem + L.flag_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);

  // weight rows of this tile: [r0a, r0a+32) and [r0b, r0b+32)
  int r0a, r0b;
  if (EPI == HM_EPI_SILU) {
    r0a = tile * kBoxRows;
    r0b = d.N / 2 + tile * kBoxRows;
  } else {
    r0a = tile * kRows;
    r0b = r0a + kBoxRows;
  }

  // 128B-swizzled TMA destinations must be 1024-byte aligned
  if (smem_u32(wsm) & 1023u) {
    if (tid == 0) report_error(d.err, HM_ERR_TIMEOUT);
    return;
  }
  // ---- prologue that touches only immutable data (weights, scales)
  if (tid == 0) {
    prefetch_tensormap(&wmap);
    for (int b = 0; b < nblk; ++b) mbar_init(&bars[b], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t pol = policy_evict_first();
    for (int b = 0; b < nblk; ++b) {
      mbar_arrive_expect_tx(&bars[b], kRows * kBlkK);
      tma_load_2d(wsm + b * (kRows * kBlkK), &wmap, k0 + b * kBlkK, r0a, &bars[b], pol);
      tma_load_2d(wsm + b * (kRows * kBlkK) + kBoxRows * kBlkK, &wmap, k0 + b * kBlkK, r0b, &bars[b], pol);
    }
  }
  if (tid < kRows) {
    const int n = tid < kBoxRows ? r0a + tid : r0b + (tid - kBoxRows);
    scale_s[tid] = n < d.N ? __half2float(reinterpret_cast<const __half*>(d.s)[n]) : 0.f;
  }
  pdl_trigger();
  // ---- everything below reads data produced by earlier launches
  pdl_wait();

  // RMSNorm inverse scales: sum of the producer's per-64-column partials in a fixed order
  for (int m = warp; m < M; m += kThreads / 32) {
    const RowRef rr = row_of(d, m);
    float inv = 0.f;
    if (rr.s->mode == HM_SRC_RMS) {
      float a = 0.f;
      for (int t = lane; t < rr.s->ss_tiles; t += 32) a += rr.s->ss[(int64_t)t * rr.s->ss_ld + rr.row];
      a = warp_sum(a);
      inv = 1.0f / sqrtf(a / static_cast<float>(rr.s->dim) + rr.s->eps);
    }
    if (lane == 0) inv_s[m] = inv;
  }
  __syncthreads();

  // activation tile [MROWS][kspan] fp16, swizzled 16-byte chunks, zero rows >= M
  {
    const int cpr = kspan / 8;
    for (int i = tid; i < MROWS * cpr; i += kThreads) {
      const int m = i / cpr, c = i - m * cpr;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (m < M) v = load_x8(d, m, k0 + 8 * c, inv_s[m], d.err);
      *reinterpret_cast<uint4*>(xsm + m * L.xp + xchunk(c) * 16) = v;
    }
  }
  __syncthreads();

  // ---- main loop: warp w owns tile rows [16w, 16w+16)
  float acc[MT][4];
#pragma unroll
  for (int j = 0; j < MT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const int g = lane >> 2, t = lane & 3;
  const int r1 = warp * 16 + g;
  bool ok = true;
  for (int b = 0; b < nblk; ++b) {
    if (!mbar_wait(&bars[b], 0, d.err)) {
      ok = false;
      break;
    }
    const uint8_t* wb = wsm + b * (kRows * kBlkK);
    const uint4 lo0 = *reinterpret_cast<const uint4*>(wb + r1 * kBlkK + (((2 * t) ^ g) << 4));
    const uint4 lo1 = *reinterpret_cast<const uint4*>(wb + r1 * kBlkK + (((2 * t + 1) ^ g) << 4));
    const uint4 hi0 = *reinterpret_cast<const uint4*>(wb + (r1 + 8) * kBlkK + (((2 * t) ^ g) << 4));
    const uint4 hi1 = *reinterpret_cast<const uint4*>(wb + (r1 + 8) * kBlkK + (((2 * t + 1) ^ g) << 4));
    const uint32_t wa[8] = {lo0.x, lo0.y, lo0.z, lo0.w, lo1.x, lo1.y, lo1.z, lo1.w};
    const uint32_t wc[8] = {hi0.x, hi0.y, hi0.z, hi0.w, hi1.x, hi1.y, hi1.z, hi1.w};
    uint32_t xw[MT][16];
#pragma unroll
    for (int j = 0; j < MT; ++j) {
      const uint8_t* xr = xsm + (8 * j + g) * L.xp;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + xchunk(16 * b + 4 * t + i) * 16);
        xw[j][4 * i + 0] = v.x;
        xw[j][4 * i + 1] = v.y;
        xw[j][4 * i + 2] = v.z;
        xw[j][4 * i + 3] = v.w;
      }
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      uint32_t a0, a1, a2, a3;
      i8x4_to_h2x2(wa[s], a0, a2);
      i8x4_to_h2x2(wc[s], a1, a3);
#pragma unroll
      for (int j = 0; j < MT; ++j) mma_16816(acc[j], a0, a1, a2, a3, xw[j][2 * s], xw[j][2 * s + 1]);
    }
  }
  if (!ok) {
    // drain: give every outstanding TMA block one more bounded chance, then leave
    for (int b = 0; b < nblk; ++b) mbar_wait(&bars[b], 0, nullptr);
    return;
  }
#pragma unroll
  for (int j = 0; j < MT; ++j) {
    const int m = 8 * j + 2 * t;
    acc_s[r1 * MP + m] = acc[j][0];
    acc_s[r1 * MP + m + 1] = acc[j][1];
    acc_s[(r1 + 8) * MP + m] = acc[j][2];
    acc_s[(r1 + 8) * MP + m + 1] = acc[j][3];
  }
  __syncthreads();

  // ---- split-K fixup: last CTA of this tile sums the partials in split order
  if (P.nsplit > 1) {
    float* ws = reinterpret_cast<float*>(d.ws);
    const int per = kRows * M;
    float* mine = ws + ((int64_t)split * P.ntiles + tile) * per;
    for (int i = tid; i < per; i += kThreads) mine[i] = acc_s[(i / M) * MP + (i % M)];
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(&d.counters[tile], 1);
      flag_s[0] = (prev == P.nsplit - 1);
    }
    __syncthreads();
    if (!flag_s[0]) return;
    __threadfence();
    for (int i = tid; i < per; i += kThreads) {
      float a = 0.f;
      for (int sp = 0; sp < P.nsplit; ++sp) a += __ldcg(ws + ((int64_t)sp * P.ntiles + tile) * per + i);
      acc_s[(i / M) * MP + (i % M)] = a;
    }
    if (tid == 0) d.counters[tile] = 0;
    __syncthreads();
  }

  // ---- epilogues
  if (EPI == HM_EPI_STORE) {
    __half* y = reinterpret_cast<__half*>(d.y);
    const __half* res = reinterpret_cast<const __half*>(d.res);
    for (int i = tid; i < kRows * M; i += kThreads) {
      const int r = i & (kRows - 1), m = i >> 6;
      const int n = r0a + r;
      float sq = 0.f;
      if (n < d.N) {
        __half v = __float2half_rn(acc_s[r * MP + m] * scale_s[r]);
        if (res) v = hadd_rn(v, res[(int64_t)m * d.ldres + n]);
        y[(int64_t)m * d.ldy + n] = v;
        const float vf = __half2float(v);
        sq = vf * vf;
      }
      sq_s[m * kRows + r] = sq;
    }
    if (d.ss_out) {
      __syncthreads();
      for (int m = warp; m < M; m += kThreads / 32) {
        const float a = warp_sum(sq_s[m * kRows + lane] + sq_s[m * kRows + lane + 32]);
        if (lane == 0) d.ss_out[(int64_t)tile * d.ss_out_ld + m] = a;
      }
    }
  } else if (EPI == HM_EPI_ROPE_KV) {
    const int hd = d.hd, qw = d.Hq * hd, kw = d.Hk * hd;
    __half* qo = reinterpret_cast<__half*>(d.q_out);
    __half* kc = reinterpret_cast<__half*>(d.kc);
    __half* vc = reinterpret_cast<__half*>(d.vc);
    for (int i = tid; i < (kRows / 2) * M; i += kThreads) {
      const int r = 2 * (i & 31), m = i >> 5;
      const int n = r0a + r;
      if (n >= d.N) continue;
      const float x0 = __half2float(__float2half_rn(acc_s[r * MP + m] * scale_s[r]));
      const float x1 = __half2float(__float2half_rn(acc_s[(r + 1) * MP + m] * scale_s[r + 1]));
      const int64_t p = d.pos[m];
      const int bb = m / d.S;
      if (p < 0 || p >= d.L || p >= d.rope_rows) {
        report_error(d.err, HM_ERR_BADINDEX);
        continue;
      }
      const int dh = n % hd;
      if (n < qw + kw) {
        const float* cs = d.rope + (p * (hd / 2) + dh / 2) * 2;
        const float c = cs[0], sn = cs[1];
        const __half y0 = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
        const __half y1 = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
        __half* dst;
        if (n < qw) {
          dst = qo + (int64_t)m * qw + n;
        } else {
          const int kh = (n - qw) / hd;
          dst = kc + (((int64_t)bb * d.Hk + kh) * d.L + p) * hd + dh;
        }
        dst[0] = y0;
        dst[1] = y1;
      } else {
        const int kh = (n - qw - kw) / hd;
        __half* dst = vc + (((int64_t)bb * d.Hk + kh) * d.L + p) * hd + dh;
        dst[0] = __float2half_rn(x0);
        dst[1] = __float2half_rn(x1);
      }
    }
  } else {  // HM_EPI_SILU
    __half* y = reinterpret_cast<__half*>(d.y);
    for (int i = tid; i < kBoxRows * M; i += kThreads) {
      const int jj = i & 31, m = i >> 5;
      const __half a = __float2half_rn(acc_s[jj * MP + m] * scale_s[jj]);
      const __half bv = __float2half_rn(acc_s[(kBoxRows + jj) * MP + m] * scale_s[kBoxRows + jj]);
      const float af = __half2float(a);
      const __half sl = __float2half_rn(__fdiv_rn(af, __fadd_rn(1.0f, expf(-af))));
      y[(int64_t)m * d.ldy + r0a + jj] = hmul_rn(sl, bv);
    }
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct MapKey {
  const void* p;
  int n, k;
  bool operator==(const MapKey& o) const { return p == o.p && n == o.n && k == o.k; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (static_cast<size_t>(k.n) * 1000003u) ^ (static_cast<size_t>(k.k) << 20);
  }
};

bool weight_map(const int8_t* w, int N, int K, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{w, N, K};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  auto enc = get_encode_fn();
  if (!enc) return false;
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  cuuint32_t box[2] = {kBlkK, kBoxRows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int ntiles_of(int N, int epi) { return epi == HM_EPI_SILU ? (N / 2) / kBoxRows : (N + kRows - 1) / kRows; }

double min_ctas_frac() {
  static double f = -1;
  if (f < 0) {
    const char* e = getenv("HM_GEMV_MIN_CTAS");
    f = e ? atof(e) : 0.6;
  }
  return f;
}

// K rounded up to whole 128-column TMA boxes (the tail is zero-filled)
int padded_k(int K) { return (K + kBlkK - 1) / kBlkK * kBlkK; }

int auto_kspan(int M, int N, int K, int epi) {
  K = padded_k(K);
  const int nt = ntiles_of(N, epi);
  const int target = static_cast<int>(min_ctas_frac() * sm_count());
  int best = 0;
  for (int ks : {1024, 512, 256, 128}) {
    if (K % ks) continue;
    best = ks;
    if (nt * (K / ks) >= target) return ks;
  }
  (void)M;
  return best;
}

template <int MT, int EPI>
cudaError_t launch_one(const CUtensorMap& map, const GemvParams& p, cudaStream_t st) {
  const SmemLayout L = smem_layout(p.kspan, 8 * MT);
  static int configured_max = 0;
  if (L.total > configured_max) {
    cudaError_t e = cudaFuncSetAttribute(gemv_i8_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_layout(kMaxKspan, 8 * MT).total);
    if (e != cudaSuccess) return e;
    configured_max = smem_layout(kMaxKspan, 8 * MT).total;
  }
  return hm_launch(gemv_i8_kernel<MT, EPI>, dim3(p.ntiles, p.nsplit), dim3(kThreads), L.total, st, p.d.pdl, map, p);
}

template <int EPI>
cudaError_t launch_mt(int mt, const CUtensorMap& map, const GemvParams& p, cudaStream_t st) {
  if (mt == 1) return launch_one<1, EPI>(map, p, st);
  if (mt == 2) return launch_one<2, EPI>(map, p, st);
  return launch_one<4, EPI>(map, p, st);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int hm_gemv_pick_kspan(int M, int N, int K, int epi, int kspan) {
  if (kspan > 0) return kspan;
  return auto_kspan(M, N, K, epi);
}

extern "C" int hm_gemv_counters(int N, int epi) { return ntiles_of(N, epi); }

extern "C" size_t hm_gemv_workspace_bytes(int M, int N, int K, int epi, int kspan) {
  const int ks = hm_gemv_pick_kspan(M, N, K, epi, kspan);
  if (ks <= 0) return 0;
  const int nsplit = padded_k(K) / ks;
  if (nsplit <= 1) return 0;
  return static_cast<size_t>(nsplit) * ntiles_of(N, epi) * kRows * M * sizeof(float);
}

extern "C" int hm_gemv_i8_fused(const hm_gemv_desc* d, hm_stream_t stream) {
  if (!d || !d->w || !d->s || d->M < 1 || d->M > kMaxM || d->N < 1 || d->K < 16 || d->K % 16) return HM_EARG;
  if (!aligned16(d->w)) return HM_EARG;
  if (d->epi == HM_EPI_SILU && (d->N % (2 * kBoxRows) || !d->y)) return HM_EARG;
  if (d->epi == HM_EPI_STORE && !d->y) return HM_EARG;
  if (d->epi == HM_EPI_STORE && d->ss_out && d->N % kRows) return HM_EARG;
  if (d->epi == HM_EPI_ROPE_KV &&
      (!d->rope || !d->pos || !d->q_out || !d->kc || !d->vc || d->hd % 64 || d->S < 1 ||
       d->N != (d->Hq + 2 * d->Hk) * d->hd))
    return HM_EARG;
  for (int i = 0; i < (d->interleave ? 2 : 1); ++i) {
    const hm_row_src& s = d->src[i];
    if (s.mode == HM_SRC_EMB) {
      if (!s.etab || !s.escale || !s.tok || (reinterpret_cast<uintptr_t>(s.etab) & 7u)) return HM_EARG;
    } else {
      if (!s.x || !aligned16(s.x) || (s.ldx % 8)) return HM_EARG;
      if (s.mode == HM_SRC_RMS && (!s.ss || !s.gamma || !aligned16(s.gamma) || s.dim <= 0)) return HM_EARG;
    }
  }
  GemvParams p;
  p.d = *d;
  const int kpad = padded_k(d->K);
  p.kspan = hm_gemv_pick_kspan(d->M, d->N, d->K, d->epi, d->kspan);
  if (p.kspan <= 0 || p.kspan > kMaxKspan || p.kspan % kBlkK || kpad % p.kspan) return HM_EARG;
  p.nsplit = kpad / p.kspan;
  p.ntiles = ntiles_of(d->N, d->epi);
  if (p.nsplit > 1) {
    if (!d->ws || !d->counters || d->n_counters < p.ntiles ||
        d->ws_bytes < static_cast<size_t>(p.nsplit) * p.ntiles * kRows * d->M * sizeof(float))
      return HM_EARG;
  }
  CUtensorMap map;
  if (!weight_map(d->w, d->N, d->K, &map)) return HM_EARG;
  const int mt = d->M <= 8 ? 1 : (d->M <= 16 ? 2 : 4);
  cudaError_t e;
  switch (d->epi) {
    case HM_EPI_STORE: e = launch_mt<HM_EPI_STORE>(mt, map, p, stream); break;
    case HM_EPI_ROPE_KV: e = launch_mt<HM_EPI_ROPE_KV>(mt, map, p, stream); break;
    case HM_EPI_SILU: e = launch_mt<HM_EPI_SILU>(mt, map, p, stream); break;
    default: return HM_EARG;
  }
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_gemv_i8(const void* x, int64_t ldx, const int8_t* w, const void* s, const void* res,
                          int64_t ldres, void* y, int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes,
                          int* counters, int n_counters, int* err, int kspan, int pdl, hm_stream_t stream) {
  hm_gemv_desc d = {};
  d.w = w;
  d.s = s;
  d.N = N;
  d.K = K;
  d.M = M;
  d.src[0].mode = HM_SRC_F16;
  d.src[0].row_mul = 1;
  d.src[0].x = x;
  d.src[0].ldx = ldx;
  d.epi = HM_EPI_STORE;
  d.y = y;
  d.ldy = ldy;
  d.res = res;
  d.ldres = ldres;
  d.ws = ws;
  d.ws_bytes = ws_bytes;
  d.counters = counters;
  d.n_counters = n_counters;
  d.err = err;
  d.kspan = kspan;
  d.pdl = pdl;
  return hm_gemv_i8_fused(&d, stream);
}

extern "C" int hm_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}

extern "C" size_t hm_abi_layout(int which) {
  switch (which) {
    case 0: return sizeof(hm_row_src);
    case 1: return sizeof(hm_gemv_desc);
    case 2: return offsetof(hm_gemv_desc, src);
    case 3: return offsetof(hm_gemv_desc, ws);
    case 4: return offsetof(hm_gemv_desc, pdl);
    default: return 0;
  }
}

extern "C" const char* hm_version(void) { return "heartmula_b200 0.1 sm_100a"; }
