// Prompt-prefill GEMM with int8 weights on the 5th-generation tensor cores (sm_100a).
//
// Replaces the M > 16 branch of the reference's `int8_mm` (app/kernels.py:46-49:
// weights dequantised to fp16, then an fp16 GEMM) for the prompt pass of the
// backbone, `Stack.__call__` -> `Block.__call__` (app/engine.py:123-153, 174-178).
//
//   C[m, n] = fp16( sum_k A[m, k] * W[n, k] * s[n] )  (+ R[m, n], rounded again)
//   SiLU epilogue (fused w1|w3): C[m, f] = fp16( fp16(silu(a)) * b ),
//                                a = fp16(acc_w1 * s), b = fp16(acc_w3 * s)
//
// int8 -> fp16 is exact, so the product over k is the same as with the
// reference's dequantised weights; the per-row scale is applied to the fp32
// sum instead of to each weight (one rounding fewer).
//
// One CTA computes a 128 x 256 output tile (for SiLU: 128 features of w1 and the
// same 128 of w3).  Warp roles:
//   warp 0      TMA producer: A tile 128x64 fp16 (128B swizzle) and the int8
//               weight tile 256x64 into a 4-stage ring.
//   warp 1      allocates 256 TMEM columns; one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) x4 per
//               k-block from shared-memory descriptors, fp32 accumulators in
//               TMEM, and releases ring slots with tcgen05.commit.
//   warps 2-9   convert the int8 tile to fp16 in the K-major 128B-swizzled
//               layout the MMA reads (double-buffered; eight warps, so two per
//               SM sub-partition hide each other's latency: with four the
//               conversion, not the MMA, set the pace), then run the epilogue:
//               tcgen05.ld of their 32 TMEM lanes (warp % 4) over half of the
//               tile's columns each, scale, round, residual/SiLU, store.
// Every wait is bounded (HM_ERR_TIMEOUT in the caller's error word).
//
// fp16-weight variant (hm_gemm_f16w): the weights come already converted to fp16 (exact
// int8 values, hm_dequant_i8_f16, made once), so TMA writes them straight into the layout
// the MMA reads, and the tiles run on SM pairs: a cluster of two CTAs computes 256 x 256 tiles with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16).  Each CTA loads its own 128 rows of A and
// its half (128 rows) of the weight tile; the leader CTA's thread issues the MMAs, which
// read both CTAs' shared memory, and its commits arrive on both CTAs' barriers.  Per SM
// that halves the weight bytes fetched from L2 per MMA: a single-SM 128 x 256 tile needs
// ~94 bytes per clock of L2 -> shared-memory fill at full tensor rate, above the ~80 B/clk
// per SM that copies reach when every SM streams at once; the pair needs ~62.
// Persistent: one CTA per SM, five 32 KB stages, two TMEM accumulators per CTA (one
// tile's epilogue overlaps the next tile's main loop).
// Products and per-element k order are the same as the int8 variant's, so are the results.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "hm_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64, NST = 4;
constexpr int kConvW = 8;                  // converter / epilogue warps
constexpr int kThreads = 64 + 32 * kConvW;  // + TMA warp + MMA warp
constexpr uint32_t kTmemCols = 256;
constexpr int kABytes = BM * BK * 2;   // 16 KB
constexpr int kBqBytes = BN * BK;      // 16 KB
constexpr int kBhBytes = BN * BK * 2;  // 32 KB

struct GemmSmem {
  uint8_t a[NST][kABytes];
  uint8_t bq[NST][kBqBytes];
  uint8_t bh[2][kBhBytes];
  uint64_t full[NST], empty[NST], bh_full[2], bh_empty[2], acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

// fp16-weight pair variant (persistent): per CTA, a ring of A (128 x 64) and weight-half
// (128 x 64) tiles, the epilogue's own staging and two sets of column scales
constexpr int NS2 = 5;
constexpr int kStageBytesP = 128 * 512;  // 128 rows x 256 fp16 results
struct GemmSmem2 {
  uint8_t a[NS2][kABytes];
  uint8_t b[NS2][kABytes];
  uint8_t stage[kStageBytesP];
  __half scl[2][256];
  uint64_t full[NS2], empty[NS2];  // full: used in the leader CTA only
  uint64_t acc_full[2], acc_empty[2];  // acc_empty: the leader's, 8 warps of each CTA arrive
  uint32_t tmem_base;
  int abort_flag;
};

struct GemmParams {
  const __half* s;
  const __half* res;
  int64_t ldr;
  __half* c;
  int64_t ldc;
  int M, N, K;  // N: output columns (features for SiLU)
  int wrows_half;  // SiLU: row offset of w3 inside W (= features)
  int ntiles;      // tiles along N (the pair kernel's tile loop)
  int n_fast;      // pair kernel: consecutive tiles walk N (1) or M (0)
  int* err;
};

// SiLU with the fast exponential and division (the value is rounded to fp16 next, so
// these differ from the IEEE forms by at most one fp16 ulp at a rounding boundary; for
// a < -87 the quotient is 0, which is also the fp16 value of silu(a) there)
HM_DEV float silu_f(float a) { return __fdividef(a, 1.f + __expf(-a)); }

// ---------------------------------------------------------------- epilogue (both kernels)
// Runs once every MMA of the tile has completed: `stage` (64 KB) holds the tile's fp16
// results, `scl` (256 values) its column scales; `release()` runs once the warp's TMEM
// reads are complete (the persistent kernel hands the accumulator back to the MMA there).
// Phase 1: the column scales (256 values) go to shared memory once; warp w (2 .. 9) reads
// TMEM lanes 32*(w%4) .. +31 (tile rows) over its part (w-2)/4 of the columns, applies
// scale (and SiLU), rounds to fp16 and stages the values (row r at 512 r bytes, 16-byte
// chunk c at slot c ^ (r & 7): conflict-free for both phases).  Phase 2: the same warp
// copies its own 32 rows out as whole 128/256-byte row segments (16-byte lanes along the
// row), adding the residual there: y = fp16(fp16(acc * s) + r), the same rounding points.
constexpr int kStageBytes = BM * 512;
template <int EPI, typename Release>
HM_DEV void epilogue_tile(const GemmParams& P, uint32_t tmem, int warp, int lane, int m_row0, int nt, uint8_t* stage,
                          __half* scl, Release release) {
  const int et = (warp - 2) * 32 + lane;  // 0 .. 255
  const int N = P.N, M = P.M;
  const int q = warp & 3, part = (warp - 2) / 4;
  constexpr int W = EPI == HM_EPI_SILU ? BN / 4 : BN / 2;  // output columns per warp
  constexpr int cpr = W / 8, rpi = 32 / cpr;              // 16-byte chunks per row, rows per copy instruction
  constexpr int kIt = 32 / rpi, kHalf = kIt / 2;           // copy instructions, in two batches
  const int col0 = EPI == HM_EPI_SILU ? nt * (BN / 2) : nt * BN;
  const __half* const R = P.res;
  // residual chunks of this lane's copy slots (row 32q + it*rpi + lane/cpr, chunk part*cpr + lane%cpr):
  // the first batch is requested now, so its latency hides behind the TMEM readout
  auto res_chunk = [&](int it) {
    const int rr = 32 * q + it * rpi + lane / cpr, m = m_row0 + rr, col = col0 + 8 * (part * cpr + lane % cpr);
    return (EPI != HM_EPI_SILU && R && m < M && col < N) ? *reinterpret_cast<const uint4*>(R + (int64_t)m * P.ldr + col)
                                                          : make_uint4(0, 0, 0, 0);
  };
  uint4 rv[kHalf];
#pragma unroll
  for (int it = 0; it < kHalf; ++it) rv[it] = res_chunk(it);
  {
    int src;
    bool ok;
    if (EPI == HM_EPI_SILU) {  // w1 scales of features nt*128 .., then w3's
      const int f = nt * (BN / 2) + (et & (BN / 2 - 1));
      src = (et < BN / 2 ? 0 : P.wrows_half) + f;
      ok = f < N;
    } else {
      src = nt * BN + et;
      ok = src < N;
    }
    scl[et] = ok ? P.s[src] : __float2half_rn(0.f);
  }
  named_bar(1, 32 * kConvW);
  const int r = 32 * q + lane;
  const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q) << 16);
  uint8_t* const srow = stage + r * 512;
#pragma unroll 1
  for (int c0 = part * W; c0 < (part + 1) * W; c0 += 16) {
    uint32_t out[8];
    if (EPI == HM_EPI_SILU) {
      float va[16], vb[16];
      tmem_ld16(trow + c0, va);
      tmem_ld16(trow + BN / 2 + c0, vb);
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        float y[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float a = __half2float(__float2half_rn(va[i + e] * __half2float(scl[c0 + i + e])));
          const float bb = __half2float(__float2half_rn(vb[i + e] * __half2float(scl[BN / 2 + c0 + i + e])));
          y[e] = __half2float(__float2half_rn(silu_f(a))) * bb;
        }
        out[i / 2] = pack_h2(y[0], y[1]);
      }
    } else {
      float v[16];
      tmem_ld16(trow + c0, v);
#pragma unroll
      for (int i = 0; i < 16; i += 2)
        out[i / 2] = pack_h2(v[i] * __half2float(scl[c0 + i]), v[i + 1] * __half2float(scl[c0 + i + 1]));
    }
    const int ch = c0 / 8;
    *reinterpret_cast<uint4*>(srow + ((ch ^ (r & 7)) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<uint4*>(srow + (((ch + 1) ^ (r & 7)) << 4)) = make_uint4(out[4], out[5], out[6], out[7]);
  }
  release();     // this warp's reads of the accumulator are complete
  __syncwarp();  // this warp's 32 rows x W columns are staged
#pragma unroll
  for (int b2 = 0; b2 < 2; ++b2) {
    if (b2 == 1) {
#pragma unroll
      for (int it = 0; it < kHalf; ++it) rv[it] = res_chunk(kHalf + it);
    }
#pragma unroll
    for (int i = 0; i < kHalf; ++i) {
      const int it = b2 * kHalf + i;
      const int rr = 32 * q + it * rpi + lane / cpr, ch = part * cpr + lane % cpr;
      const int m = m_row0 + rr, col = col0 + 8 * ch;
      const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 512 + ((ch ^ (rr & 7)) << 4));
      if (m < M && col < N) {
        uint4 y = v;
        if (EPI != HM_EPI_SILU && R) {
          const uint32_t* a = &v.x;
          const uint32_t* b = &rv[i].x;
          uint32_t* o = &y.x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(a + e));
            const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(b + e));
            o[e] = pack_h2(fa.x + fb.x, fa.y + fb.y);
          }
        }
        *reinterpret_cast<uint4*>(P.c + (int64_t)m * P.ldc + col) = y;
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_i8w_kernel(const __grid_constant__ CUtensorMap amap,
                                                               const __grid_constant__ CUtensorMap wmap,
                                                               const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * BM;
  const int nt = blockIdx.y;
  const int nk = P.K / BK;
  int* const err = P.err;

  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < NST; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1 + kConvW);  // MMA commit (A consumed) + the converter warps (int8 tile consumed)
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.bh_full[i], kConvW);
      mbar_init(&sm.bh_empty[i], 1);
    }
    mbar_init(&sm.acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_s = &sm.abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&amap);
      prefetch_tensormap(&wmap);
      const int r0 = EPI == HM_EPI_SILU ? nt * (BN / 2) : nt * BN;
      const int r1 = EPI == HM_EPI_SILU ? P.wrows_half + nt * (BN / 2) : nt * BN + BN / 2;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % NST;
        if (kb >= NST) mbar_wait_ab(&sm.empty[s], ((kb / NST) - 1) & 1, err, abort_s);
        mbar_arrive_expect_tx(&sm.full[s], kABytes + kBqBytes);
        tma_load_2d_plain(sm.a[s], &amap, kb * BK, m0, &sm.full[s]);
        tma_load_2d_plain(sm.bq[s], &wmap, kb * BK, r0, &sm.full[s]);
        tma_load_2d_plain(sm.bq[s] + kBqBytes / 2, &wmap, kb * BK, r1, &sm.full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN);
      const uint64_t a0 = sw128_desc(smem_u32(sm.a[0])), b0 = sw128_desc(smem_u32(sm.bh[0]));
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % NST, b = kb & 1;
        mbar_wait_ab(&sm.full[s], (kb / NST) & 1, err, abort_s);
        mbar_wait_ab(&sm.bh_full[b], (kb >> 1) & 1, err, abort_s);
        tc_fence_after();
        const uint64_t ad = a0 + s * (kABytes >> 4), bd = b0 + b * (kBhBytes >> 4);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)  // +32 bytes per K=16 step inside the 128-byte swizzle row
          umma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
        umma_commit(&sm.empty[s]);
        umma_commit(&sm.bh_empty[b]);
      }
      umma_commit(&sm.acc_full);
    }
  } else {
    // ------------------------------------------------------------ converters, then epilogue
    const int ct = tid - 64;  // 0 .. 32 * kConvW - 1
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % NST, b = kb & 1;
      mbar_wait_ab(&sm.full[s], (kb / NST) & 1, err, abort_s);
      if (kb >= 2) mbar_wait_ab(&sm.bh_empty[b], ((kb >> 1) - 1) & 1, err, abort_s);
      const uint8_t* src = sm.bq[s];
      uint8_t* dst = sm.bh[b];
#pragma unroll
      for (int i = 0; i < (BN * BK / 16) / (32 * kConvW); ++i) {
        const int id = ct + 32 * kConvW * i;  // 16-byte int8 chunk: row n, k = 16j .. 16j+15
        const int n = id >> 2, j = id & 3;
        const uint4 q = *reinterpret_cast<const uint4*>(src + n * BK + j * 16);
        uint4 h0, h1;
        i8x4_to_h2x2(q.x, h0.x, h0.y);
        i8x4_to_h2x2(q.y, h0.z, h0.w);
        i8x4_to_h2x2(q.z, h1.x, h1.y);
        i8x4_to_h2x2(q.w, h1.z, h1.w);
        uint8_t* row = dst + (n >> 3) * 1024 + (n & 7) * 128;
        *reinterpret_cast<uint4*>(row + (((2 * j) ^ (n & 7)) << 4)) = h0;
        *reinterpret_cast<uint4*>(row + (((2 * j + 1) ^ (n & 7)) << 4)) = h1;
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.bh_full[b]);
        mbar_arrive(&sm.empty[s]);
      }
    }
    mbar_wait_ab(&sm.acc_full, 0, err, abort_s);
    tc_fence_after();
    epilogue_tile<EPI>(P, tmem, warp, lane, m0, nt, sm.a[0], reinterpret_cast<__half*>(sm.bq[0]), [] {});
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// fp16 weights on SM pairs, persistent: cluster c (two CTAs along M, one per SM) computes
// the 256 x 256 tiles c, c + clusters, ...; tile t = (M pair, N tile) with consecutive
// tiles walking N when the activations are the larger operand (the tiles in flight then
// share a few M pairs of A and all of W, both L2-resident; w2's A is 134 MB at 8 x 1024
// tokens), else walking M; rows pair*256 + rank*128 .. +127 in CTA `rank`, columns
// nt*256 .. +255 (SiLU: features nt*128 .. +127 of w1 and of w3).  Two 256-column TMEM
// accumulators per CTA: the MMA fills one while the epilogue warps of both CTAs drain the
// other.
template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_f16w_pair_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                          const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  GemmSmem2& sm = *reinterpret_cast<GemmSmem2*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int mpairs = (P.M + 2 * BM - 1) / (2 * BM), T = mpairs * P.ntiles;
  const int nk = P.K / BK;
  int* const err = P.err;

  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < NS2; ++i) {
      mbar_init(&sm.full[i], 1);   // the leader's producer (expect_tx) + both CTAs' copies (bytes)
      mbar_init(&sm.empty[i], 1);  // the leader's MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);             // the leader's MMA commit
      mbar_init(&sm.acc_empty[i], 2 * kConvW);   // every epilogue warp of both CTAs
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(&sm.tmem_base, 2 * BN);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_s = &sm.abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tensormap(&amap);
      prefetch_tensormap(&wmap);
      const uint32_t full0 = dsmem_addr(&sm.full[0], 0);  // the leader's ring barriers
      int g = 0;  // k-blocks over all of this pair's tiles
      for (int t = pair; t < T; t += npairs) {
        const int mp = P.n_fast ? t / P.ntiles : t % mpairs, nt = P.n_fast ? t % P.ntiles : t / mpairs;
        const int m_row0 = mp * 2 * BM + static_cast<int>(rank) * BM;
        const int brow = EPI == HM_EPI_SILU ? (rank == 0 ? 0 : P.wrows_half) + nt * (BN / 2)
                                            : nt * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % NS2;
          if (g >= NS2) mbar_wait_ab(&sm.empty[s], ((g / NS2) - 1) & 1, err, abort_s);
          if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 4 * kABytes);  // A + B halves of both CTAs
          tma_load_2d_pair(sm.a[s], &amap, kb * BK, m_row0, full0 + 8 * s);
          tma_load_2d_pair(sm.b[s], &wmap, kb * BK, brow, full0 + 8 * s);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16(2 * BM, BN);
      const uint64_t a0 = sw128_desc(smem_u32(sm.a[0])), b0 = sw128_desc(smem_u32(sm.b[0]));
      int g = 0, i = 0;
      for (int t = pair; t < T; t += npairs, ++i) {
        const int ab = i & 1;
        // the accumulator's previous tile has been read out by both CTAs' epilogues
        if (i >= 2 && !*abort_s && !mbar_wait_cluster(&sm.acc_empty[ab], ((i >> 1) - 1) & 1, err)) *abort_s = 1;
        tc_fence_after();
        const uint32_t acc = tmem + ab * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % NS2;
          mbar_wait_ab(&sm.full[s], (g / NS2) & 1, err, abort_s);
          tc_fence_after();
          const uint64_t ad = a0 + s * (kABytes >> 4), bd = b0 + s * (kABytes >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_f16_pair(acc, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair(&sm.empty[s]);
        }
        umma_commit_pair(&sm.acc_full[ab]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs: their 128 rows)
    const uint32_t acc_empty0 = dsmem_addr(&sm.acc_empty[0], 0);  // the leader's
    int i = 0;
    for (int t = pair; t < T; t += npairs, ++i) {
      const int ab = i & 1;
      const int mp = P.n_fast ? t / P.ntiles : t % mpairs, nt = P.n_fast ? t % P.ntiles : t / mpairs;
      const int m_row0 = mp * 2 * BM + static_cast<int>(rank) * BM;
      mbar_wait_ab(&sm.acc_full[ab], (i >> 1) & 1, err, abort_s);
      tc_fence_after();
      epilogue_tile<EPI>(P, tmem + ab * BN, warp, lane, m_row0, nt, sm.stage, sm.scl[ab], [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0)
            mbar_arrive(&sm.acc_empty[ab]);
          else
            mbar_arrive_dsmem(acc_empty0 + 8 * ab);
        }
      });
    }
  }
  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the pair's copies, MMAs or commits may touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
}

static_assert(sizeof(GemmSmem::a) >= kStageBytes && sizeof(GemmSmem::bq) >= 512, "epilogue staging space (int8 kernel)");
static_assert(kStageBytesP >= kStageBytes, "epilogue staging space (pair kernel)");

// ---------------------------------------------------------------- host side
struct MapKey {
  const void* p;
  int64_t rows, cols, ld;
  int kind;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld && kind == o.kind;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (std::hash<int64_t>()(k.rows) * 31) ^ (std::hash<int64_t>()(k.ld) * 17) ^
           static_cast<size_t>(k.kind);
  }
};

// kind 0: fp16 activations [rows, cols] (row stride ld elements), box 64 x 128, 128B swizzle
// kind 1: int8 weights [rows, cols] (row stride cols bytes), box 64 x 128, no swizzle
bool tile_map(const void* p, int64_t rows, int64_t cols, int64_t ld, int kind, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{p, rows, cols, ld, kind};
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
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r;
  if (kind == 0) {
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[2] = {BK, BM};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
    cuuint32_t box[2] = {BK, BN / 2};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

template <int EPI>
cudaError_t launch_gemm(const CUtensorMap& am, const CUtensorMap& wm, const GemmParams& p, int ntiles_n, bool wf16,
                        hm_stream_t st) {
  const size_t smem = (wf16 ? sizeof(GemmSmem2) : sizeof(GemmSmem)) + 1024;
  static bool configured[2] = {false, false};
  if (!configured[wf16]) {
    cudaError_t e = wf16 ? cudaFuncSetAttribute(gemm_f16w_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem))
                         : cudaFuncSetAttribute(gemm_i8w_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[wf16] = true;
  }
  if (wf16) {  // persistent: one cluster of two CTAs per pair of SMs, at most one per tile
    static int sms = 0;
    if (sms == 0) {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                    cudaSuccess)
        return cudaErrorInvalidValue;
    }
    GemmParams q = p;
    q.ntiles = ntiles_n;
    q.n_fast = p.M > (EPI == HM_EPI_SILU ? 2 * p.N : p.N);  // A (M x K) larger than W (rows x K)
    const int64_t tiles = (int64_t)((p.M + 2 * BM - 1) / (2 * BM)) * ntiles_n;
    const int pairs = static_cast<int>(tiles < sms / 2 ? tiles : sms / 2);
    return hm_launch(gemm_f16w_pair_kernel<EPI>, dim3(2 * pairs), dim3(kThreads), smem, st, false, am, wm, q);
  }
  const dim3 grid((p.M + BM - 1) / BM, ntiles_n);
  return hm_launch(gemm_i8w_kernel<EPI>, grid, dim3(kThreads), smem, st, false, am, wm, p);
}

// Shared argument checks and launch of both variants (wf16: w holds fp16 [N, K]).
int gemm_entry(const void* a, int64_t lda, const void* w, bool wf16, const void* s, const void* res, int64_t ldr,
               void* c, int64_t ldc, int M, int N, int K, int epi, int* err, hm_stream_t stream) {
  if (!a || !w || !s || !c || M < 1 || N < 1 || K < BK || K % BK != 0) return HM_EARG;
  if (epi != HM_EPI_STORE && epi != HM_EPI_SILU) return HM_EARG;
  if (epi == HM_EPI_SILU && (res != nullptr || N % 2 != 0)) return HM_EARG;
  const int nout = epi == HM_EPI_SILU ? N / 2 : N;  // output columns
  // 16-byte vector stores / loads of 16-column groups and TMA stride rules
  if (nout % 16 != 0 || lda % 8 != 0 || ldc % 8 != 0 || lda < K || ldc < nout) return HM_EARG;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(c)) & 15u) return HM_EARG;
  if (res && (ldr % 8 != 0 || ldr < N || (reinterpret_cast<uintptr_t>(res) & 15u))) return HM_EARG;
  if (reinterpret_cast<uintptr_t>(w) & 15u) return HM_EARG;
  CUtensorMap am, wm;
  if (!tile_map(a, M, K, lda, 0, &am) || !tile_map(w, N, K, K, wf16 ? 0 : 1, &wm)) return HM_EARG;
  GemmParams p;
  p.s = reinterpret_cast<const __half*>(s);
  p.res = reinterpret_cast<const __half*>(res);
  p.ldr = ldr;
  p.c = reinterpret_cast<__half*>(c);
  p.ldc = ldc;
  p.M = M;
  p.N = nout;
  p.K = K;
  p.wrows_half = epi == HM_EPI_SILU ? N / 2 : 0;
  p.ntiles = 0;
  p.n_fast = 0;
  p.err = err;
  const int tn = epi == HM_EPI_SILU ? (nout + BN / 2 - 1) / (BN / 2) : (N + BN - 1) / BN;
  const cudaError_t e = epi == HM_EPI_SILU ? launch_gemm<HM_EPI_SILU>(am, wm, p, tn, wf16, stream)
                                           : launch_gemm<HM_EPI_STORE>(am, wm, p, tn, wf16, stream);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

}  // namespace

extern "C" int hm_gemm_i8w(const void* a, int64_t lda, const int8_t* w, const void* s, const void* res,
                           int64_t ldr, void* c, int64_t ldc, int M, int N, int K, int epi, int* err,
                           hm_stream_t stream) {
  return gemm_entry(a, lda, w, false, s, res, ldr, c, ldc, M, N, K, epi, err, stream);
}

extern "C" int hm_gemm_f16w(const void* a, int64_t lda, const void* w, const void* s, const void* res, int64_t ldr,
                            void* c, int64_t ldc, int M, int N, int K, int epi, int* err, hm_stream_t stream) {
  return gemm_entry(a, lda, w, true, s, res, ldr, c, ldc, M, N, K, epi, err, stream);
}
