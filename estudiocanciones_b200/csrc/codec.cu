// HeartCodec detokenize on sm_100a: the implicit-GEMM convolution that carries every
// GEMM-shaped layer of the codec, and the small fused kernels around it.
//
// Replaces, in the reference's codec (app/heartcodec/**, driven by app/codec_lite.py:63-75):
//   * nn.Linear and ProjectLayer's Conv1d(k=3) of the flow-matching LlamaTransformer
//     (models/transformer.py:153-167, 205-220, 235-250, 300-375) with their bias, the
//     ProjectLayer scale, RoPE of q/k (:112-127), the gated residuals of the ada-norm
//     blocks (:185-201) and the SiLU-gated MLP (:160-162);
//   * Conv1d / ConvTranspose1d / PReLU / residual adds of ScalarModel.decode
//     (models/sq_codec.py:33-105 convolutions, :133-147 PostProcessor, :150-172
//     ResidualUnit, :204-245 ResDecoderBlock, :506-510 decode).
//
// conv_gemm_kernel computes, for batch item b, output row t and column n,
//   acc[b, t, n] = sum_{j < taps} sum_{c < cin} x[b, t + off0 + j*dil, c] * w[j, n, c]
// with rows of x outside [0, tin) read as zero.  A Conv1d is taps = k, off0 = -left
// padding, dil = dilation; a Linear is taps = 1; a causal ConvTranspose1d with
// kernel 2s is taps = 2 (off0 = 0, dil = -1) over s*Cout columns (output phase-major,
// which is the time-major [s*T, Cout] layout itself); the PostProcessor's nearest
// repeat followed by a causal conv folds into taps over the unrepeated rows.  The
// host lays the weights out for that (estudiocanciones_b200/codec.py).
//
// Tensor-core mapping: M = 128 output rows of one batch item, N = BN (64/128/256)
// columns, K walked as (tap, 64-channel chunk).  Each K step is one 3-D TMA box of x
// ({64 channels, 128 rows, 1 item}, the row coordinate shifted by the tap offset; TMA
// zero-fills outside the item's rows, which is the convolution's zero padding and keeps
// items apart) and one 2-D box of w, 128B-swizzled, into a ring of stages;
// tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) x4 per stage with fp32
// accumulators in TMEM.  Persistent CTAs (one per SM) walk the tiles column-fastest;
// two TMEM accumulators let one tile's epilogue overlap the next tile's MMAs.
// Warps: 0 TMA producer, 1 TMEM allocation + MMA issue (one thread), 2-9 epilogue
// (two warps per TMEM lane quarter, each half of the tile's columns).
// Every wait is bounded (HM_ERR_TIMEOUT in the caller's error word).
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "heartmula_b200.h"
#include "hm_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kEpiW = 8;
constexpr int kThr = 64 + 32 * kEpiW;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kSmemBudget = 192 * 1024;

template <int BN>
struct CCfg {
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int NST = kSmemBudget / (kABytes + kBBytes);  // 4 / 6 / 8 stages
};

template <int BN>
struct ConvSmem {
  uint8_t a[CCfg<BN>::NST][kABytes];
  uint8_t b[CCfg<BN>::NST][CCfg<BN>::kBBytes];
  float stg[kEpiW][32 * 32];  // per epilogue warp: 32 rows x 32 columns in flight to global memory
  uint64_t full[CCfg<BN>::NST], empty[CCfg<BN>::NST], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct ConvP {
  int B, T, N, npad, nkc, taps, off0, dil, mtiles, ntiles, tiles;
  const float* bias;
  float scale, prelu;
  int act, epi, y_f32, rope_cols, hd;
  const void* res;
  int64_t res_ld;
  const float* gate;
  int64_t gate_ld;
  const float2* rope;
  void* y;
  int64_t y_ld;
  int* err;
};

HM_DEV void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

HM_DEV float silu_fast(float a) { return __fdividef(a, 1.f + __expf(-a)); }

HM_DEV float act_of(float v, int act, float prelu) {
  if (act == HM_ACT_PRELU) return v >= 0.f ? v : prelu * v;
  if (act == HM_ACT_SILU) return silu_fast(v);
  return v;
}

struct TileIdx {
  int nt, mt, b;
};
HM_DEV TileIdx tile_of(const ConvP& P, int tt) {
  TileIdx r;
  r.nt = tt % P.ntiles;
  const int rest = tt / P.ntiles;
  r.mt = rest % P.mtiles;
  r.b = rest / P.mtiles;
  return r;
}

// Copy-out of one staged 32 x 32 chunk (rows t0 .. t0+31 of item b, columns n0 .. n0+31) with
// the residual / gate epilogues, along rows in 16-byte lanes.  Rows past T are skipped; a
// chunk that crosses N goes per element.
HM_DEV void conv_copy_out(const ConvP& P, const float* stg, int64_t row0, int t0, int b, int n0) {
  const int lane = threadIdx.x & 31;
  const bool full_cols = n0 + 32 <= P.N;
  if (full_cols) {
    // whole chunk: the residual (and gate) loads of every pass are issued before any store, so
    // their latencies overlap (the output may alias the residual, which keeps the compiler from
    // moving a load above an earlier store)
    if (P.y_f32) {  // lane = (row 4i + lane/8, columns 4 (lane%8) ..)
      const int c = (lane & 7) * 4, n = n0 + c;
      float4 gv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (P.epi == HM_CEPI_GATED) gv = *reinterpret_cast<const float4*>(P.gate + static_cast<int64_t>(b) * P.gate_ld + n);
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // two batches of four passes (registers)
        float4 rv[4];
        if (P.epi == HM_CEPI_GATED) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 4 * (4 * half + i) + (lane >> 3);
            rv[i] = t0 + rr < P.T ? *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(P.res) +
                                                                     (row0 + rr) * P.res_ld + n)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = 4 * (4 * half + i) + (lane >> 3);
          if (t0 + rr >= P.T) continue;
          float4 f = *reinterpret_cast<const float4*>(stg + rr * 32 + (((c >> 2) ^ (rr & 7)) << 2));
          if (P.epi == HM_CEPI_GATED) {
            f.x = rv[i].x + gv.x * f.x;
            f.y = rv[i].y + gv.y * f.y;
            f.z = rv[i].z + gv.z * f.z;
            f.w = rv[i].w + gv.w * f.w;
          }
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(P.y) + (row0 + rr) * P.y_ld + n) = f;
        }
      }
    } else {  // fp16: lane = (row 8i + lane/4, columns 8 (lane%4) ..)
      const int c = (lane & 3) * 8, n = n0 + c;
      uint4 rv[4];
      if (P.epi == HM_CEPI_RES) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = 8 * i + (lane >> 2);
          rv[i] = t0 + rr < P.T
                      ? *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(P.res) + (row0 + rr) * P.res_ld + n)
                      : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = 8 * i + (lane >> 2);
        if (t0 + rr >= P.T) continue;
        const float* sr = stg + rr * 32;
        const float4 f0 = *reinterpret_cast<const float4*>(sr + ((((c >> 2)) ^ (rr & 7)) << 2));
        const float4 f1 = *reinterpret_cast<const float4*>(sr + ((((c >> 2) + 1) ^ (rr & 7)) << 2));
        float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        if (P.epi == HM_CEPI_RES) {
          const __half2* h2 = reinterpret_cast<const __half2*>(&rv[i]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 r2 = __half22float2(h2[e]);
            v[2 * e] += r2.x;
            v[2 * e + 1] += r2.y;
          }
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(P.y) + (row0 + rr) * P.y_ld + n) =
            make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]), pack_h2(v[4], v[5]), pack_h2(v[6], v[7]));
      }
    }
    return;
  }
  // a chunk past N: per element, lane = row, columns n0 .. N-1
  const int rr = lane;
  if (t0 + rr >= P.T) return;
  const int64_t row = row0 + rr;
  for (int e = 0; e < 32 && n0 + e < P.N; ++e) {
    float x = stg[rr * 32 + ((((e >> 2)) ^ (rr & 7)) << 2) + (e & 3)];
    const int n = n0 + e;
    if (P.epi == HM_CEPI_GATED)
      x = reinterpret_cast<const float*>(P.res)[row * P.res_ld + n] + P.gate[static_cast<int64_t>(b) * P.gate_ld + n] * x;
    else if (P.epi == HM_CEPI_RES)
      x += __half2float(reinterpret_cast<const __half*>(P.res)[row * P.res_ld + n]);
    if (P.y_f32)
      reinterpret_cast<float*>(P.y)[row * P.y_ld + n] = x;
    else
      reinterpret_cast<__half*>(P.y)[row * P.y_ld + n] = __float2half_rn(x);
  }
}

// Epilogue of one tile row: this thread's TMEM lane (output row t of item b) over its half h of
// the tile's columns (SiLU-mul: a quarter of the features), bias / scale / activation and the
// epilogue variant, then the stores.  Warp-collective (tcgen05.ld): every lane of the warp calls it.
template <int BN>
HM_DEV void conv_epilogue(const ConvP& P, uint32_t tb, int nt, int b, int t, int h, float* stg) {
  const bool valid = t < P.T;
  const int64_t row = static_cast<int64_t>(b) * P.T + t;
  if (P.epi == HM_CEPI_SILU) {
    // weight rows in blocks of 256: 128 gate rows then the same 128 features' up rows;
    // this warp: features h*64 .. h*64+63 of the block (BN == 256)
    for (int f0 = h * (BN / 4); f0 < (h + 1) * (BN / 4); f0 += 16) {
      float gv[16], uv[16], o[32];
      tmem_ld16(tb + f0, gv);
      tmem_ld16(tb + BN / 2 + f0, uv);
      const int ng = nt * BN + f0, nu = ng + BN / 2;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        float a = gv[e], u = uv[e];
        if (P.bias) {
          a += P.bias[ng + e];
          u += P.bias[nu + e];
        }
        o[e] = silu_fast(a * P.scale) * (u * P.scale);
      }
      if (valid) {
        const int f = nt * (BN / 2) + f0;  // output feature
        __half* y = reinterpret_cast<__half*>(P.y) + row * P.y_ld + f;
        *reinterpret_cast<uint4*>(y) = make_uint4(pack_h2(o[0], o[1]), pack_h2(o[2], o[3]), pack_h2(o[4], o[5]),
                                                  pack_h2(o[6], o[7]));
        *reinterpret_cast<uint4*>(y + 8) = make_uint4(pack_h2(o[8], o[9]), pack_h2(o[10], o[11]),
                                                      pack_h2(o[12], o[13]), pack_h2(o[14], o[15]));
      }
    }
  } else {
    // per 32-column chunk: bias, scale, activation and RoPE in registers (this thread's row),
    // then the chunk goes through the warp's staging buffer so that the residual / gate
    // reads and the stores run along rows (16-byte lanes), not one row per lane
    const int lane = threadIdx.x & 31;
    const int t0 = t - lane;  // the warp's first row
    const int64_t row0 = static_cast<int64_t>(b) * P.T + t0;
    for (int c0 = h * (BN / 2); c0 < (h + 1) * (BN / 2); c0 += 32) {
      uint32_t raw[32];
      tmem_ld32_nowait(tb + c0, raw);
      tmem_wait_ld();
      const int n0 = nt * BN + c0;
      if (n0 >= P.N) continue;  // uniform over the warp
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float a = __uint_as_float(raw[e]);
        if (P.bias && n0 + e < P.N) a += P.bias[n0 + e];
        v[e] = act_of(a * P.scale, P.act, P.prelu);
      }
      if (P.epi == HM_CEPI_ROPE && n0 < P.rope_cols && valid) {
        // pairs (n, n+1), n even, rotated by the angle of (t, (n % hd) / 2)
        const float2* tab = P.rope + static_cast<int64_t>(t) * (P.hd / 2) + (n0 % P.hd) / 2;
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 cs = tab[e / 2];
          const float x1 = v[e], x2 = v[e + 1];
          v[e] = x1 * cs.x - x2 * cs.y;
          v[e + 1] = x1 * cs.y + x2 * cs.x;
        }
      }
      // row `lane` of the chunk: float4 q at slot q ^ (lane & 7) (four lanes per bank group)
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(stg + lane * 32 + ((q ^ (lane & 7)) << 2)) =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      __syncwarp();
      conv_copy_out(P, stg, row0, t0, b, n0);
      __syncwarp();
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThr, 1)
    conv_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ ConvP P) {
  constexpr int NST = CCfg<BN>::NST;
  constexpr int kBB = CCfg<BN>::kBBytes;
  extern __shared__ uint8_t smem_raw[];
  ConvSmem<BN>& sm = *reinterpret_cast<ConvSmem<BN>*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int* const err = P.err;
  const int nk = P.taps * P.nkc;

  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < NST; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kEpiW);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_s = &sm.abort_flag;
  pdl_wait();  // the previous launch's outputs (this launch's inputs) are complete
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
      int g = 0;
      for (int tt = blockIdx.x; tt < P.tiles; tt += gridDim.x) {
        const TileIdx ti = tile_of(P, tt);
        const int t0 = ti.mt * kBM;
        for (int j = 0; j < P.taps; ++j) {
          const int xrow = t0 + P.off0 + j * P.dil;
          const int wrow = j * P.npad + ti.nt * BN;
          for (int kc = 0; kc < P.nkc; ++kc, ++g) {
            const int s = g % NST;
            if (g >= NST) mbar_wait_ab(&sm.empty[s], ((g / NST) - 1) & 1, err, abort_s);
            mbar_arrive_expect_tx(&sm.full[s], kABytes + kBB);
            tma_load_3d(sm.a[s], &xmap, kc * kBK, xrow, ti.b, &sm.full[s]);
            tma_load_2d_plain(sm.b[s], &wmap, kc * kBK, wrow, &sm.full[s]);
          }
        }
      }
      // every copy issued has landed before the CTA's shared memory can be released
      for (int t = g > NST ? g - NST : 0; t < g; ++t) mbar_wait(&sm.full[t % NST], (t / NST) & 1, err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, BN);
      const uint64_t a0 = sw128_desc(smem_u32(sm.a[0])), b0 = sw128_desc(smem_u32(sm.b[0]));
      int g = 0, i = 0;
      for (int tt = blockIdx.x; tt < P.tiles; tt += gridDim.x, ++i) {
        const int ab = i & 1;
        if (i >= 2) mbar_wait_ab(&sm.acc_empty[ab], ((i >> 1) - 1) & 1, err, abort_s);
        tc_fence_after();
        const uint32_t acc = tmem + ab * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % NST;
          mbar_wait_ab(&sm.full[s], (g / NST) & 1, err, abort_s);
          tc_fence_after();
          const uint64_t ad = a0 + s * (kABytes >> 4), bd = b0 + s * (kBB >> 4);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) umma_f16(acc, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&sm.empty[s]);
        }
        umma_commit(&sm.acc_full[ab]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q4 = warp & 3;         // TMEM lane quarter this warp may read
    const int h = (warp - 2) >> 2;   // column half of the tile
    const int r = 32 * q4 + lane;    // tile row = TMEM lane
    int i = 0;
    for (int tt = blockIdx.x; tt < P.tiles; tt += gridDim.x, ++i) {
      const int ab = i & 1;
      const TileIdx ti = tile_of(P, tt);
      const int t = ti.mt * kBM + r;
      mbar_wait_ab(&sm.acc_full[ab], (i >> 1) & 1, err, abort_s);
      tc_fence_after();
      const uint32_t tb = tmem + (static_cast<uint32_t>(32 * q4) << 16) + ab * BN;
      conv_epilogue<BN>(P, tb, ti.nt, ti.b, t, h, sm.stg[warp - 2]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// ---------------------------------------------------------------- SM-pair variant
// The same GEMM on pairs of SMs (a cluster of two CTAs, tcgen05 cta_group::2): a pair
// computes 256 output rows x BN columns, each CTA loading its own 128 rows of x and its half
// (BN/2 rows) of the weight tile by TMA (no multicast), the loads completing on the leader
// CTA's barriers; the leader's thread issues tcgen05.mma.cta_group::2 (M=256, N=BN, K=16),
// which reads both CTAs' shared memory, with fp32 accumulators in each CTA's TMEM (its 128
// rows x BN columns), and its commits (multicast to both CTAs) free the ring slots and
// signal finished tiles.  Per SM this halves the weight bytes streamed from L2 per MMA flop.
// Tiles: 256-row blocks of one item (rank r takes rows 128 r .. of the block) x BN columns.
template <int BN>
struct PairCfg {
  static constexpr int kBH = (BN / 2) * kBK * 2;  // this CTA's half of a weight stage
  static constexpr int NST = kSmemBudget / (kABytes + kBH);  // 8 (bn 128) / 6 (bn 256) stages
};

template <int BN>
struct PairSmem {
  uint8_t a[PairCfg<BN>::NST][kABytes];
  uint8_t b[PairCfg<BN>::NST][PairCfg<BN>::kBH];
  float stg[kEpiW][32 * 32];  // per epilogue warp: 32 rows x 32 columns in flight to global memory
  uint64_t full[PairCfg<BN>::NST], empty[PairCfg<BN>::NST];  // full: used in the leader only
  uint64_t acc_full[2], acc_empty[2];  // acc_empty: the leader's, both CTAs' epilogue warps arrive
  uint32_t tmem_base;
  int abort_flag;
};

HM_DEV void tma_load_3d_pair(void* dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThr, 1)
    conv_gemm_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                          const __grid_constant__ ConvP P) {
  constexpr int NST = PairCfg<BN>::NST;
  constexpr int kBH = PairCfg<BN>::kBH;
  extern __shared__ uint8_t smem_raw[];
  PairSmem<BN>& sm = *reinterpret_cast<PairSmem<BN>*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  int* const err = P.err;
  const int nk = P.taps * P.nkc;

  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < NST; ++i) {
      mbar_init(&sm.full[i], 1);   // the leader's producer (expect_tx) + both CTAs' copies (bytes)
      mbar_init(&sm.empty[i], 1);  // the leader's MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);            // the leader's MMA commit
      mbar_init(&sm.acc_empty[i], 2 * kEpiW);   // every epilogue warp of both CTAs
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(&sm.tmem_base, 2 * BN);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_s = &sm.abort_flag;
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
      const uint32_t full0 = dsmem_addr(&sm.full[0], 0);  // the leader's ring barriers
      int g = 0;
      for (int tt = pair; tt < P.tiles; tt += npairs) {
        const TileIdx ti = tile_of(P, tt);
        const int t0 = ti.mt * 2 * kBM + static_cast<int>(rank) * kBM;
        for (int j = 0; j < P.taps; ++j) {
          const int xrow = t0 + P.off0 + j * P.dil;
          const int wrow = j * P.npad + ti.nt * BN + static_cast<int>(rank) * (BN / 2);
          for (int kc = 0; kc < P.nkc; ++kc, ++g) {
            const int s = g % NST;
            if (g >= NST) mbar_wait_ab(&sm.empty[s], ((g / NST) - 1) & 1, err, abort_s);
            if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 2 * (kABytes + kBH));  // both CTAs' loads
            tma_load_3d_pair(sm.a[s], &xmap, kc * kBK, xrow, ti.b, full0 + 8 * s);
            tma_load_2d_pair(sm.b[s], &wmap, kc * kBK, wrow, full0 + 8 * s);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16(2 * kBM, BN);
      const uint64_t a0 = sw128_desc(smem_u32(sm.a[0])), b0 = sw128_desc(smem_u32(sm.b[0]));
      int g = 0, i = 0;
      for (int tt = pair; tt < P.tiles; tt += npairs, ++i) {
        const int ab = i & 1;
        // the accumulator's previous tile has been read out by both CTAs' epilogues
        if (i >= 2 && !*abort_s && !mbar_wait_cluster(&sm.acc_empty[ab], ((i >> 1) - 1) & 1, err)) *abort_s = 1;
        tc_fence_after();
        const uint32_t acc = tmem + ab * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % NST;
          mbar_wait_ab(&sm.full[s], (g / NST) & 1, err, abort_s);
          tc_fence_after();
          const uint64_t ad = a0 + s * (kABytes >> 4), bd = b0 + s * (kBH >> 4);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) umma_f16_pair(acc, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair(&sm.empty[s]);
        }
        umma_commit_pair(&sm.acc_full[ab]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs: their 128 rows)
    const uint32_t acc_empty0 = dsmem_addr(&sm.acc_empty[0], 0);  // the leader's
    const int q4 = warp & 3, h = (warp - 2) >> 2, r = 32 * q4 + lane;
    int i = 0;
    for (int tt = pair; tt < P.tiles; tt += npairs, ++i) {
      const int ab = i & 1;
      const TileIdx ti = tile_of(P, tt);
      const int t = ti.mt * 2 * kBM + static_cast<int>(rank) * kBM + r;
      mbar_wait_ab(&sm.acc_full[ab], (i >> 1) & 1, err, abort_s);
      tc_fence_after();
      const uint32_t tb = tmem + (static_cast<uint32_t>(32 * q4) << 16) + ab * BN;
      conv_epilogue<BN>(P, tb, ti.nt, ti.b, t, h, sm.stg[warp - 2]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&sm.acc_empty[ab]);
        else
          mbar_arrive_dsmem(acc_empty0 + 8 * ab);
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the pair's copies, MMAs or commits may touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
}

// ---------------------------------------------------------------- tensor maps
struct MapKey {
  const void* p;
  int64_t d0, d1, d2, s1, s2;
  int box1;
  bool operator==(const MapKey& o) const {
    return p == o.p && d0 == o.d0 && d1 == o.d1 && d2 == o.d2 && s1 == o.s1 && s2 == o.s2 && box1 == o.box1;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (std::hash<int64_t>()(k.d1) * 31) ^ (std::hash<int64_t>()(k.s1) * 17) ^
           (std::hash<int64_t>()(k.d2) * 7) ^ static_cast<size_t>(k.box1);
  }
};

// fp16 tensor of rank 2 {d0 (contiguous), d1} or 3 {d0, d1, d2} with byte strides s1 (, s2); box
// {64, box1 (, 1)}, 128B swizzle, zero fill outside.
bool conv_map(int rank, const void* p, int64_t d0, int64_t d1, int64_t d2, int64_t s1, int64_t s2, int box1,
              CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{p, d0, d1, rank == 3 ? d2 : -1, s1, s2, box1};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  auto enc = hm_encode_fn();
  if (!enc) return false;
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1), static_cast<cuuint64_t>(s2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box1), 1};
  cuuint32_t es[3] = {1, 1, 1};
  if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(p), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 8192) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

int sm_count_cached() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  return sms;
}

template <int BN>
cudaError_t launch_conv(const CUtensorMap& xm, const CUtensorMap& wm, ConvP p, hm_stream_t st) {
  const size_t smem = sizeof(ConvSmem<BN>) + 1024;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e =
        cudaFuncSetAttribute(conv_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  p.ntiles = p.npad / BN;
  p.tiles = p.B * p.mtiles * p.ntiles;
  const int sms = sm_count_cached();
  const int grid = p.tiles < sms ? p.tiles : sms;
  return hm_launch(conv_gemm_kernel<BN>, dim3(grid), dim3(kThr), smem, st, 1, xm, wm, p);
}

template <int BN>
cudaError_t launch_conv_pair(const CUtensorMap& xm, const CUtensorMap& wm, ConvP p, hm_stream_t st) {
  const size_t smem = sizeof(PairSmem<BN>) + 1024;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(conv_gemm_pair_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  p.mtiles = (p.T + 2 * kBM - 1) / (2 * kBM);  // 256-row blocks per item
  p.ntiles = p.npad / BN;
  p.tiles = p.B * p.mtiles * p.ntiles;
  const int pairs_avail = sm_count_cached() / 2;
  const int pairs = p.tiles < pairs_avail ? p.tiles : pairs_avail;
  return hm_launch(conv_gemm_pair_kernel<BN>, dim3(2 * pairs), dim3(kThr), smem, st, 0, xm, wm, p);
}

// Tile width by a cost model: waves of tiles over the SMs times the time of one tile's
// 64-wide k step, relative to bn = 256: 0.68 for bn = 128 and 0.55 for bn = 64 (measured on
// the codec's shapes, 2 x 744 rows: with a whole wave of tiles each width is bound by its
// shared-memory fill, bytes per MMA flop falling with the width).  Ties go to the wider tile.
int pick_bn(const hm_conv_desc* d, int mtiles) {
  const int64_t sms = sm_count_cached();
  const int64_t rows = static_cast<int64_t>(d->B) * mtiles;
  int best = 0;
  double best_cost = 0.0;
  for (int bn : {256, 128, 64}) {
    if (d->npad % bn) continue;
    const int64_t tiles = rows * (d->npad / bn);
    const double step = bn == 256 ? 1.0 : (bn == 128 ? 0.68 : 0.55);
    const double cost = static_cast<double>((tiles + sms - 1) / sms) * step;
    if (best == 0 || cost < best_cost * 0.999) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

// ---------------------------------------------------------------- small kernels
// RMSNorm (weight w) or LayerNorm (no affine) of one fp32 row, then the ada-norm
// modulation: out = fp16( norm(x) * (1 + scale[b]) + shift[b] ).
__global__ void __launch_bounds__(256) norm_mod_kernel(const float* __restrict__ x, int64_t ldx,
                                                       const float* __restrict__ w, const float* __restrict__ shift,
                                                       const float* __restrict__ scale, int64_t mod_ld,
                                                       __half* __restrict__ out, int64_t ldo, int T, int D, float eps,
                                                       int layer_norm) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int b = static_cast<int>(row / T);
  const float* xr = x + row * ldx;
  __shared__ float red[2][8];
  const int wid = threadIdx.x >> 5, ln = threadIdx.x & 31, nw = static_cast<int>(blockDim.x >> 5);
  // LayerNorm: mean first, then the mean square of x - mean (two passes over the row);
  // RMSNorm: the mean square of x
  float mean = 0.f;
  if (layer_norm) {
    float s1 = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) s1 += xr[i];
    s1 = warp_sum(s1);
    if (ln == 0) red[0][wid] = s1;
    __syncthreads();
    float t1 = 0.f;
    for (int k = 0; k < nw; ++k) t1 += red[0][k];
    mean = t1 / D;
  }
  float s2 = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = xr[i] - mean;
    s2 += v * v;
  }
  s2 = warp_sum(s2);
  if (ln == 0) red[1][wid] = s2;
  __syncthreads();
  float t2 = 0.f;
  for (int k = 0; k < nw; ++k) t2 += red[1][k];
  const float inv = rsqrtf(t2 / D + eps);
  const float* sh = shift + static_cast<int64_t>(b) * mod_ld;
  const float* sc = scale + static_cast<int64_t>(b) * mod_ld;
  __half* o = out + row * ldo;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = (xr[i] - mean) * inv;
    if (w) v *= w[i];
    o[i] = __float2half_rn(v * (1.f + sc[i]) + sh[i]);
  }
}

// The same with the row in registers: D / 8 threads (whole warps), 8 values each (two 16-byte
// loads of x, one 16-byte store), D % 256 == 0 and 16-byte aligned rows.
__global__ void __launch_bounds__(1024) norm_mod8_kernel(const float* __restrict__ x, int64_t ldx,
                                                         const float* __restrict__ w, const float* __restrict__ shift,
                                                         const float* __restrict__ scale, int64_t mod_ld,
                                                         __half* __restrict__ out, int64_t ldo, int T, int D,
                                                         float eps, int layer_norm) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int b = static_cast<int>(row / T);
  const int c0 = 8 * threadIdx.x;
  __shared__ float red[2][32];
  const int wid = threadIdx.x >> 5, ln = threadIdx.x & 31, nw = static_cast<int>((blockDim.x + 31) >> 5);
  const float4* xr = reinterpret_cast<const float4*>(x + row * ldx + c0);
  const float4 a0 = xr[0], a1 = xr[1];
  float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  float mean = 0.f;
  if (layer_norm) {
    float s1 = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    s1 = warp_sum(s1);
    if (ln == 0) red[0][wid] = s1;
    __syncthreads();
    float t1 = 0.f;
    for (int k = 0; k < nw; ++k) t1 += red[0][k];
    mean = t1 / D;
  }
  float s2 = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    v[e] -= mean;
    s2 += v[e] * v[e];
  }
  s2 = warp_sum(s2);
  if (ln == 0) red[1][wid] = s2;
  __syncthreads();
  float t2 = 0.f;
  for (int k = 0; k < nw; ++k) t2 += red[1][k];
  const float inv = rsqrtf(t2 / D + eps);
  const float* sh = shift + static_cast<int64_t>(b) * mod_ld + c0;
  const float* sc = scale + static_cast<int64_t>(b) * mod_ld + c0;
  float o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float u = v[e] * inv;
    if (w) u *= w[c0 + e];
    o[e] = u * (1.f + sc[e]) + sh[e];
  }
  *reinterpret_cast<uint4*>(out + row * ldo + c0) =
      make_uint4(pack_h2(o[0], o[1]), pack_h2(o[2], o[3]), pack_h2(o[4], o[5]), pack_h2(o[6], o[7]));
}

// Residual-VQ code lookup + project_out: out[t, :] = fp16( W (sum_q cb[q][codes[q, t]]) + bias ).
// One CTA per frame; codes outside [0, K) are clamped to it, as the codec wrapper clamps its
// input (app/codec_lite.py:72).
__global__ void __launch_bounds__(256) vq_embed_kernel(const int64_t* __restrict__ codes, int64_t ld_codes, int nq,
                                                       const float* __restrict__ cb, int K, int cd,
                                                       const float* __restrict__ pw, const float* __restrict__ pb,
                                                       __half* __restrict__ out, int64_t ldo, int dim) {
  extern __shared__ float vsum[];  // [cd]
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < cd; c += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < nq; ++q) {
      int64_t id = codes[static_cast<int64_t>(q) * ld_codes + t];
      id = id < 0 ? 0 : (id >= K ? K - 1 : id);
      s += cb[(static_cast<int64_t>(q) * K + id) * cd + c];
    }
    vsum[c] = s;
  }
  __syncthreads();
  for (int n = threadIdx.x; n < dim; n += blockDim.x) {
    const float* wr = pw + static_cast<int64_t>(n) * cd;
    float a = pb ? pb[n] : 0.f;
    for (int c = 0; c < cd; ++c) a = fmaf(wr[c], vsum[c], a);
    out[static_cast<int64_t>(t) * ldo + n] = __float2half_rn(a);
  }
}

// dst row (rep*t + i) = src row t, i < rep (nearest-neighbour upsampling along time).
__global__ void upsample_rows_kernel(const __half* __restrict__ src, int64_t lds, int rows, int cols, int rep,
                                     __half* __restrict__ dst, int64_t ldd) {
  const int64_t total = static_cast<int64_t>(rows) * rep * cols;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e % cols);
    const int64_t orow = e / cols;
    dst[orow * ldd + c] = src[(orow / rep) * lds + c];
  }
}

// One Euler step of the flow-matching ODE and the next step's estimator input.
//   v == NULL: x = noise (the initial latents)
//   else     : x += dt * (u + g (c - u))  (nb == 2: u = rows [0,T), c = rows [T,2T) of v), or x += dt * v
//   then rows < L_in of x take the in-context blend (1 - (1 - 1e-6) t_next) noise + t_next inc
//   (last step: final == 1, rows < L_in = inc), and unless final the fp16 copy of x goes to
//   columns [0, C) of the nb estimator-input item rows (the first call also writes the
//   in-context latents, inc rows < L_in and zeros after, to columns [C, 2C)).
__global__ void euler_kernel(const float* __restrict__ v, int nb, float* __restrict__ x,
                             const float* __restrict__ noise, const float* __restrict__ inc, int T, int C, int L_in,
                             float dt, float g, float t_next, int final, __half* __restrict__ xin, int64_t ldx,
                             int64_t xin_bstride) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = static_cast<int64_t>(T) * C;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / C);
    float xv;
    if (!v) {
      xv = noise[e];
    } else {
      float d = v[e];
      if (nb == 2) d = d + g * (v[e + total] - d);
      xv = x[e] + dt * d;
    }
    if (t < L_in) xv = final ? inc[e] : (1.f - (1.f - 1e-6f) * t_next) * noise[e] + t_next * inc[e];
    x[e] = xv;
    if (!final) {
      const int c = static_cast<int>(e % C);
      const __half hv = __float2half_rn(xv);
      // the first call (v == NULL) also writes the in-context columns [C, 2C): inc rows < L_in, else 0
      const __half hi = __float2half_rn(t < L_in ? inc[e] : 0.f);
      for (int b = 0; b < nb; ++b) {
        __half* row = xin + b * xin_bstride + static_cast<int64_t>(t) * ldx;
        row[c] = hv;
        if (!v) row[C + c] = hi;
      }
    }
  }
}

// Latent [T, nband*Cb] (fp32) -> the scalar decoder's input bands [nband, T, Cb] (fp16),
// quantised as round(9 x) / 9 (round half to even).
__global__ void band_quant_kernel(const float* __restrict__ x, int T, int Cb, int nband, __half* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(T) * Cb * nband;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e % Cb);
    const int64_t rest = e / Cb;
    const int t = static_cast<int>(rest % T), k = static_cast<int>(rest / T);
    const float xv = x[static_cast<int64_t>(t) * (nband * Cb) + k * Cb + c];
    out[e] = __float2half_rn(rintf(9.f * xv) / 9.f);
  }
}

// Timestep-embedding tail: act = fp16(silu(E)) (the ada-norm linear's input) and the output
// norm's modulation shift = tab[0] + E, scale = tab[1] + E.
__global__ void temb_post_kernel(const float* __restrict__ E, int S, int D, const float* __restrict__ tab,
                                 __half* __restrict__ act, float* __restrict__ shift, float* __restrict__ scale) {
  const int64_t total = static_cast<int64_t>(S) * D;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(e % D);
    const float v = E[e];
    act[e] = __float2half_rn(v / (1.f + expf(-v)));
    shift[e] = tab[d] + v;
    scale[e] = tab[D + d] + v;
  }
}

// Window output assembly: out[c][start + i] = cur[c][i], cross-faded over the first ovlp
// samples with w_i = i / (ovlp - 1) (w_{ovlp-1} = 1): out = out (1 - w) + cur w, in fp64.
__global__ void overlap_add_kernel(const float* __restrict__ cur, int64_t cur_ld, float* __restrict__ out,
                                   int64_t out_ld, int C, int64_t start, int64_t n, int64_t ovlp) {
  const int64_t total = static_cast<int64_t>(C) * n;
  const double step = ovlp > 1 ? 1.0 / static_cast<double>(ovlp - 1) : 0.0;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e / n);
    const int64_t i = e % n;
    const float cv = cur[c * cur_ld + i];
    float* o = out + c * out_ld + start + i;
    if (i < ovlp) {
      const double w = i == ovlp - 1 ? 1.0 : static_cast<double>(i) * step;
      *o = static_cast<float>(static_cast<double>(*o) * (1.0 - w) + static_cast<double>(cv) * w);
    } else {
      *o = cv;
    }
  }
}

unsigned grid_for(int64_t total, int threads) {
  const int64_t want = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count_cached()) * 16;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int hm_conv1d_gemm(const hm_conv_desc* d, hm_stream_t stream) {
  if (!d || !d->x || !d->w || !d->y) return HM_EARG;
  if (d->B < 1 || d->T < 1 || d->tin < 1 || d->cin < kBK || d->cin % kBK || d->N < 1 || d->taps < 1 ||
      d->npad < d->N || d->npad % 64)
    return HM_EARG;
  if (d->act < HM_ACT_NONE || d->act > HM_ACT_SILU || d->epi < HM_CEPI_STORE || d->epi > HM_CEPI_ROPE) return HM_EARG;
  if (!al16(d->x) || !al16(d->w) || !al16(d->y) || d->x_ld % 8 || d->x_bstride % 8 || d->x_ld < d->cin) return HM_EARG;
  const int64_t span = static_cast<int64_t>(d->taps - 1) * (d->dil < 0 ? -d->dil : d->dil);
  if (span > (1 << 20) || d->off0 < -(1 << 20) || d->off0 > (1 << 20)) return HM_EARG;
  if (d->T > (1 << 30) - kBM - (1 << 21) || d->tin > (1 << 30)) return HM_EARG;
  const int out_cols = d->epi == HM_CEPI_SILU ? d->N / 2 : d->N;
  // 16-byte vector stores of whole 32-column groups (outputs of fewer columns are stored per element)
  if (d->y_ld < out_cols || (out_cols >= 32 && d->y_ld % (d->y_f32 ? 4 : 8))) return HM_EARG;
  if (d->epi == HM_CEPI_SILU && d->y_ld % 8) return HM_EARG;
  if (d->epi == HM_CEPI_SILU && (d->N % 256 || d->npad != d->N || d->y_f32)) return HM_EARG;
  if (d->epi == HM_CEPI_GATED && (!d->res || !d->gate || !d->y_f32)) return HM_EARG;
  if (d->epi == HM_CEPI_RES && (!d->res || d->y_f32)) return HM_EARG;
  // 16-byte residual / gate loads along rows (outputs of fewer than 32 columns go per element)
  if (out_cols >= 32 && d->epi == HM_CEPI_GATED && (!al16(d->res) || d->res_ld % 4 || !al16(d->gate) || d->gate_ld % 4))
    return HM_EARG;
  if (out_cols >= 32 && d->epi == HM_CEPI_RES && (!al16(d->res) || d->res_ld % 8)) return HM_EARG;
  if (d->epi == HM_CEPI_ROPE && (!d->rope || d->hd < 2 || d->hd % 64 || d->rope_cols % d->hd)) return HM_EARG;
  const int mtiles = (d->T + kBM - 1) / kBM;
  // bn > 0: single-SM tiles of that width; -128 / -256: SM-pair tiles (256 rows) of that width;
  // 0: SM pairs of 256 columns where they measured faster (K >= 3072 and at least two waves of
  // pair tiles: the codec's second-stage q|k|v and gate|up, 3-9 %), else the tile-width model
  bool pair = d->bn < 0;
  if (d->bn == 0 && d->npad % 256 == 0 && static_cast<int64_t>(d->cin) * d->taps >= 3072) {
    const int64_t ptiles = static_cast<int64_t>(d->B) * ((d->T + 2 * kBM - 1) / (2 * kBM)) * (d->npad / 256);
    pair = ptiles >= sm_count_cached();
  }
  int bn = d->bn < 0 ? -d->bn
                     : (pair || d->epi == HM_CEPI_SILU ? 256 : (d->bn > 0 ? d->bn : pick_bn(d, mtiles)));
  if (pair ? (bn != 128 && bn != 256) : (bn != 64 && bn != 128 && bn != 256)) return HM_EARG;
  if (d->npad % bn || (d->epi == HM_CEPI_SILU && bn != 256)) return HM_EARG;
  CUtensorMap xm, wm;
  // x as {cin, tin, B} (an item's rows zero-fill past its ends); one item: any valid item stride
  const int64_t xb = d->B > 1 ? d->x_bstride : static_cast<int64_t>(d->tin) * d->x_ld;
  if (d->B > 1 && d->x_bstride < static_cast<int64_t>(d->tin) * d->x_ld) return HM_EARG;
  if (!conv_map(3, d->x, d->cin, d->tin, d->B, d->x_ld * 2, xb * 2, kBM, &xm)) return HM_EARG;
  if (!conv_map(2, d->w, d->cin, static_cast<int64_t>(d->taps) * d->npad, 1, static_cast<int64_t>(d->cin) * 2, 0,
                pair ? bn / 2 : bn, &wm))
    return HM_EARG;
  ConvP p;
  p.B = d->B;
  p.T = d->T;
  p.N = d->N;
  p.npad = d->npad;
  p.nkc = d->cin / kBK;
  p.taps = d->taps;
  p.off0 = d->off0;
  p.dil = d->dil;
  p.mtiles = mtiles;
  p.ntiles = p.tiles = 0;
  p.bias = d->bias;
  p.scale = d->scale;
  p.prelu = d->prelu;
  p.act = d->act;
  p.epi = d->epi;
  p.y_f32 = d->y_f32;
  p.rope_cols = d->rope_cols;
  p.hd = d->hd;
  p.res = d->res;
  p.res_ld = d->res_ld;
  p.gate = d->gate;
  p.gate_ld = d->gate_ld;
  p.rope = reinterpret_cast<const float2*>(d->rope);
  p.y = d->y;
  p.y_ld = d->y_ld;
  p.err = d->err;
  cudaError_t e;
  if (pair)
    e = bn == 256 ? launch_conv_pair<256>(xm, wm, p, stream) : launch_conv_pair<128>(xm, wm, p, stream);
  else if (bn == 256)
    e = launch_conv<256>(xm, wm, p, stream);
  else if (bn == 128)
    e = launch_conv<128>(xm, wm, p, stream);
  else
    e = launch_conv<64>(xm, wm, p, stream);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_norm_mod(const float* x, int64_t ldx, const float* w, const float* shift, const float* scale,
                                 int64_t mod_ld, void* out, int64_t ldo, int B, int T, int D, float eps,
                                 int layer_norm, hm_stream_t stream) {
  if (!x || !shift || !scale || !out || B < 1 || T < 1 || D < 1 || ldx < D || ldo < D) return HM_EARG;
  // whole warps (the reductions shuffle over full warps): D % 256 == 0
  const bool vec = D % 256 == 0 && D / 8 <= 1024 && ldx % 4 == 0 && ldo % 8 == 0 && mod_ld % 4 == 0 && al16(x) &&
                   al16(out) && al16(shift) && al16(scale);
  if (vec) {
    const cudaError_t e = hm_launch(norm_mod8_kernel, dim3(static_cast<unsigned>(B) * T), dim3(D / 8), 0, stream, 1, x,
                                    ldx, w, shift, scale, mod_ld, reinterpret_cast<__half*>(out), ldo, T, D, eps,
                                    layer_norm);
    return e == cudaSuccess ? HM_OK : static_cast<int>(e);
  }
  const cudaError_t e = hm_launch(norm_mod_kernel, dim3(static_cast<unsigned>(B) * T), dim3(256), 0, stream, 1, x, ldx,
                                  w, shift, scale, mod_ld, reinterpret_cast<__half*>(out), ldo, T, D, eps, layer_norm);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_vq_embed(const int64_t* codes, int64_t ld_codes, int nq, int Tc, const float* codebooks, int K,
                                 int cd, const float* proj_w, const float* proj_b, void* out, int64_t ldo, int dim,
                                 hm_stream_t stream) {
  if (!codes || !codebooks || !proj_w || !out || nq < 1 || Tc < 1 || K < 1 || cd < 1 || cd > 1024 || dim < 1 ||
      ldo < dim || ld_codes < Tc)
    return HM_EARG;
  vq_embed_kernel<<<Tc, 256, cd * sizeof(float), stream>>>(codes, ld_codes, nq, codebooks, K, cd, proj_w, proj_b,
                                                           reinterpret_cast<__half*>(out), ldo, dim);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_upsample_rows(const void* src, int64_t lds, int rows, int cols, int rep, void* dst,
                                      int64_t ldd, hm_stream_t stream) {
  if (!src || !dst || rows < 1 || cols < 1 || rep < 1 || lds < cols || ldd < cols) return HM_EARG;
  const int64_t total = static_cast<int64_t>(rows) * rep * cols;
  upsample_rows_kernel<<<grid_for(total, 256), 256, 0, stream>>>(reinterpret_cast<const __half*>(src), lds, rows, cols,
                                                                 rep, reinterpret_cast<__half*>(dst), ldd);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_euler(const float* v, int nb, float* x, const float* noise, const float* inc, int T, int C,
                              int L_in, float dt, float g, float t_next, int final, void* xin, int64_t ldx,
                              int64_t xin_bstride, hm_stream_t stream) {
  if (!x || !noise || (L_in > 0 && !inc) || (nb != 1 && nb != 2) || T < 1 || C < 1 || L_in < 0 || L_in > T ||
      (!final && (!xin || ldx < 2 * C)))
    return HM_EARG;
  const int64_t total = static_cast<int64_t>(T) * C;
  const cudaError_t e = hm_launch(euler_kernel, dim3(grid_for(total, 256)), dim3(256), 0, stream, 1, v, nb, x, noise,
                                  inc, T, C, L_in, dt, g, t_next, final, reinterpret_cast<__half*>(xin), ldx,
                                  xin_bstride);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_band_quant(const float* x, int T, int Cb, int nband, void* out, hm_stream_t stream) {
  if (!x || !out || T < 1 || Cb < 1 || nband < 1) return HM_EARG;
  const int64_t total = static_cast<int64_t>(T) * Cb * nband;
  band_quant_kernel<<<grid_for(total, 256), 256, 0, stream>>>(x, T, Cb, nband, reinterpret_cast<__half*>(out));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_temb_post(const float* E, int S, int D, const float* tab, void* act, float* shift,
                                  float* scale, hm_stream_t stream) {
  if (!E || !tab || !act || !shift || !scale || S < 1 || D < 1) return HM_EARG;
  const int64_t total = static_cast<int64_t>(S) * D;
  temb_post_kernel<<<grid_for(total, 256), 256, 0, stream>>>(E, S, D, tab, reinterpret_cast<__half*>(act), shift,
                                                             scale);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_codec_overlap_add(const float* cur, int64_t cur_ld, float* out, int64_t out_ld, int C, int64_t start,
                                    int64_t n, int64_t ovlp, hm_stream_t stream) {
  if (!cur || !out || C < 1 || n < 0 || start < 0 || ovlp < 0 || ovlp > n || cur_ld < n || out_ld < start + n)
    return HM_EARG;
  if (n == 0) return HM_OK;
  const int64_t total = static_cast<int64_t>(C) * n;
  overlap_add_kernel<<<grid_for(total, 256), 256, 0, stream>>>(cur, cur_ld, out, out_ld, C, start, n, ovlp);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
