// Persistent stage runner: a whole chain of decode launches as ONE cooperative
// kernel (sm_100a).
//
// A decode frame is a chain of small dependent steps (per layer: the fused
// qkv GEMV, attention, o GEMV, w1|w3 GEMV, w2 GEMV; the heads; the embedding
// sums) that the reference issues as separate launches inside one CUDA graph
// (app/engine.py:180-211, 328-354, 409-461).  At 8 rows every step is short, so
// per-launch start-up (empty weight pipeline, activation staging) dominates.
// Here a sequence of such steps ("stages") runs in one persistent kernel with
// one CTA per SM:
//
//  * a producer warp streams the int8 weights of every GEMV stage of the
//    sequence through a 10-stage TMA ring, running ahead across stage
//    boundaries (weights never depend on activations), so the HBM stream does
//    not stop while the CTAs synchronise;
//  * four consumer warps execute the stages in order, separated by a grid-wide
//    barrier (one counter, release/acquire, bounded spin); the GEMV stages are
//    the same tiles, prologues (RMSNorm / embedding gather) and epilogues
//    (residual + sum of squares, RoPE + KV write, SiLU·mul) as hm_gemv_i8_fused,
//    the attention stages the tensor-core split-K decode attention of
//    hm_decode_attn (head_dim 128), with its split merge by the last CTA;
//  * the launch is cooperative, so all CTAs are co-resident and the barrier
//    cannot deadlock; every wait is bounded and a timeout sets HM_ERR_TIMEOUT
//    and a sequence-wide abort flag that releases every later wait.
//
// Constraints of a stage (checked when it is added): GEMV with at most 8 rows
// whose activations (all of K) fit the shared-memory region; attention with
// head_dim 128 and G <= 8; embedding sums with D % 16 == 0.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "hm_common.cuh"

namespace {

constexpr int kTileRows = 16;
constexpr int kBox = 128;
constexpr int kBoxBytes = kTileRows * kBox;
constexpr int kStage = 4 * kBoxBytes;  // 8 KB: four 16x128 weight boxes
constexpr int kRing = 10;              // weight ring stages
constexpr int kCons = 256;             // 8 consumer warps
constexpr int kCW = kCons / 32;
constexpr int kThreads = kCons + 32;
constexpr int kBarCons = 1;            // named barrier of all consumer warps; 2, 3: attention groups
constexpr int kRows = 8;               // activation rows per GEMV stage
constexpr int kMP = kRows + 1;
constexpr int kXRegion = 139776;       // activations of 8 rows x K=8192 (+pitch pad), or 2 attention groups
constexpr int kMaxSplit = 32;
constexpr int kMaxG = 8;
constexpr int kTcPos = 64;
constexpr int kTcNst = 2;              // K/V stages per attention group
constexpr int kTcBox = kTcPos * 128;

enum StageType : int { ST_GEMV = 0, ST_ATTN = 1, ST_EMBSUM = 2 };

struct GemvStage {
  hm_gemv_desc d;
  int rt, ks, kspan, per_tile, ntiles, has_gamma, keep;
};

struct AttnStage {
  const __half* q;
  const int64_t* pos;
  __half* o;
  int R, S, Hq, Hk, L, nsplit;
  float scale;
  float* ws;
  int* counters;
};

struct EmbStage {
  const int64_t* tok;
  int64_t tok_ld;
  int ncb;
  int64_t vocab;
  const int8_t* tab;
  const __half* scale;
  int64_t rows;
  int R, D;
  __half* x;
  float* ss;
  int64_t ss_ld;
};

struct alignas(64) Stage {
  CUtensorMap map0;  // GEMV: weights; ATTN: K cache
  CUtensorMap map1;  // ATTN: V cache
  int type;
  int pad_[15];
  union {
    GemvStage g;
    AttnStage a;
    EmbStage e;
  } u;
};

struct SeqCtl {
  const Stage* stages;
  int n;
  unsigned* barrier;  // zeroed before each launch
  int* abort;         // sequence-wide abort flag (zeroed before each launch)
  int* err;
};

// attention buffers of one group of 4 warps (two groups inside the activation region)
struct TcSmem {
  uint8_t k[kTcNst][2][kTcBox];
  uint8_t v[kTcNst][2][kTcBox];
  float mw[4][kMaxG], lw[4][kMaxG];
  float cw[kMaxG][kMaxSplit], cl[kMaxG][kMaxSplit], cden[kMaxG];
  int flag;
};
constexpr int kTcBytes = (sizeof(TcSmem) + 1023) / 1024 * 1024;
static_assert(2 * kTcBytes <= kXRegion, "attention buffers exceed the activation region");

struct Smem {
  uint8_t ring[kRing][kStage];  // 1024-aligned (offset 0)
  uint8_t xr[kXRegion];         // activations (+ gammas) or TcSmem; 1024-aligned
  float red[kCW * kTileRows * kMP];
  float inv[kRows], esc[kRows];
  const uint8_t* rowp[kRows];
  int rmode[kRows], rsel[kRows];
  uint64_t full[kRing], empty[kRing], xbar, abar[2][kTcNst];
  int abort_local;
};

HM_DEV uint32_t ld_acquire_u32(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
HM_DEV void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t swz(const uint8_t* box, int row, int chunk) {
  return smem_u32(box + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ---------------------------------------------------------------- grid barrier
// Arrive after stage s, wait for every CTA's arrival before stage s+1.  Bounded:
// after HM_WAIT_NS the waiter records HM_ERR_TIMEOUT, raises the sequence abort
// flag (so every other wait gives up at once) and carries on.
__device__ void grid_arrive(const SeqCtl& c, int tid) {
  fence_proxy_async_smem();  // this thread's generic writes to shared memory before later async-proxy writes
  named_bar(kBarCons, kCons);
  if (tid == 0) {
    __threadfence();
    red_release_add(c.barrier, 1u);
  }
}

__device__ void grid_wait(const SeqCtl& c, unsigned target, int tid) {
  if (tid == 0) {
    volatile int* ab = c.abort;
    if (ld_acquire_u32(c.barrier) < target && !*ab) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t i = 0;; ++i) {
        if (ld_acquire_u32(c.barrier) >= target) break;
        if ((i & 63u) == 0) {
          if (*ab) break;
          if (globaltimer_ns() - t0 > HM_WAIT_NS) {
            report_error(c.err, HM_ERR_TIMEOUT);
            *ab = 1;
            break;
          }
        }
      }
    }
    fence_proxy_async_global();  // later bulk/TMA reads of data other CTAs wrote
  }
  named_bar(kBarCons, kCons);
}

// ---------------------------------------------------------------- producer
__device__ void producer(const SeqCtl& c, Smem& sm) {
  const uint64_t pol_first = policy_evict_first();
  const uint64_t pol_last = policy_evict_last();
  volatile int* ab = &sm.abort_local;
  int it = 0;
  for (int s = 0; s < c.n; ++s) {
    const Stage* st = c.stages + s;
    if (st->type != ST_GEMV) continue;
    const GemvStage& g = st->u.g;
    const int rt = g.rt, ks = g.ks, per_tile = g.per_tile, ntiles = g.ntiles;
    const int half_n = g.d.N / 2;
    const uint64_t pol = g.keep ? pol_last : pol_first;
    const CUtensorMap* map = &st->map0;
    prefetch_tensormap(map);
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      for (int j = 0; j < per_tile; ++j, ++it) {
        const int slot = it % kRing;
        if (it >= kRing) mbar_wait_ab(&sm.empty[slot], ((it / kRing) - 1) & 1, c.err, ab);
        const int kx = j * ks;
        mbar_arrive_expect_tx(&sm.full[slot], kStage);
#pragma unroll
        for (int b = 0; b < 4; ++b)
          tma_load_2d(sm.ring[slot] + b * kBoxBytes, map, kx + (b / rt) * kBox,
                      (rt == 2 && (b % 2) == 1 ? half_n : 0) + tile * kTileRows, &sm.full[slot], pol);
      }
    }
  }
}

// ---------------------------------------------------------------- GEMV stage
__device__ __forceinline__ const hm_row_src& src_of(const hm_gemv_desc& d, int m, int& row, int& sel) {
  sel = d.interleave ? (m & 1) : 0;
  const int local = d.interleave ? (m >> 1) : m;
  const hm_row_src& s = d.src[sel];
  row = local * s.row_mul + s.row_add;
  return s;
}

__device__ void gemv_stage(const Stage* st, Smem& sm, int& it, uint32_t& xuse, int* err) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile int* ab = &sm.abort_local;
  const GemvStage& G = st->u.g;
  if ((int)blockIdx.x >= G.ntiles) return;  // no tile here: nothing to stage (uniform over the CTA)
  const hm_gemv_desc& d = G.d;
  const int K = d.K, N = d.N, M = d.M, epi = d.epi;
  const int rt = G.rt, ks = G.ks, kspan = G.kspan, per_tile = G.per_tile, ntiles = G.ntiles;
  const int xp = kspan * 2 + 16;
  uint8_t* xsm = sm.xr;
  __half* gam_s = reinterpret_cast<__half*>(sm.xr + kRows * xp);
  const bool has_gamma = G.has_gamma != 0;

  if (tid < kRows) {
    const int m = tid;
    int mode = -1, sel = 0;
    const uint8_t* base = nullptr;
    float esc = 0.f;
    if (m < M) {
      int row;
      const hm_row_src& s = src_of(d, m, row, sel);
      mode = s.mode;
      if (mode == HM_SRC_EMB) {
        const int64_t id = s.tok[(int64_t)row * s.tok_ld + s.tok_col] + s.tok_off;
        if (id < 0 || id >= s.erows) {
          report_error(err, HM_ERR_BADINDEX);
          mode = -1;
        } else {
          base = reinterpret_cast<const uint8_t*>(s.etab + id * (int64_t)K);
          esc = __half2float(reinterpret_cast<const __half*>(s.escale)[id]);
        }
      } else {
        base = reinterpret_cast<const uint8_t*>(reinterpret_cast<const __half*>(s.x) + (int64_t)row * s.ldx);
      }
    }
    sm.rmode[m] = mode;
    sm.rsel[m] = sel;
    sm.rowp[m] = base;
    sm.esc[m] = esc;
  }
  const bool g0 = has_gamma && d.src[0].mode == HM_SRC_RMS;
  const bool g1 = has_gamma && d.interleave && d.src[1].mode == HM_SRC_RMS;
  named_bar(kBarCons, kCons);

  // ---- stage activations: bulk copy per fp16/RMS row and per gamma, cp.async for embedding rows
  const int cpr = kspan / 8;
  if (tid == 0) {
    uint32_t bytes = 0;
    for (int m = 0; m < M; ++m) bytes += (sm.rmode[m] == HM_SRC_F16 || sm.rmode[m] == HM_SRC_RMS) ? K * 2 : 0;
    bytes += (g0 ? K * 2 : 0) + (g1 ? K * 2 : 0);
    mbar_arrive_expect_tx(&sm.xbar, bytes);
    for (int m = 0; m < M; ++m)
      if (sm.rmode[m] == HM_SRC_F16 || sm.rmode[m] == HM_SRC_RMS) bulk_load(xsm + m * xp, sm.rowp[m], K * 2, &sm.xbar);
    if (g0) bulk_load(gam_s, d.src[0].gamma, K * 2, &sm.xbar);
    if (g1) bulk_load(gam_s + kspan, d.src[1].gamma, K * 2, &sm.xbar);
  }
  for (int m = 0; m < kRows; ++m) {
    const int mode = m < M ? sm.rmode[m] : -1;
    const uint8_t* base = sm.rowp[m];
    uint8_t* xr = xsm + m * xp;
    for (int c = tid; c < cpr; c += kCons) {
      if (mode < 0 || 8 * c >= K)
        *reinterpret_cast<uint4*>(xr + c * 16) = make_uint4(0, 0, 0, 0);
      else if (mode == HM_SRC_EMB)
        cp_async8(xr + c * 16, base + 8 * c);
    }
  }
  for (int m = warp; m < M; m += kCons / 32) {
    int row, sel;
    const hm_row_src& s = src_of(d, m, row, sel);
    if (s.mode != HM_SRC_RMS) continue;
    const float* ss = s.ss;
    const int tiles = s.ss_tiles;
    const int64_t ld = s.ss_ld;
    const float dim = static_cast<float>(s.dim), eps = s.eps;
    const float a = warp_sum_partials(ss, tiles, ld, row, lane);
    if (lane == 0) sm.inv[m] = 1.0f / sqrtf(a / dim + eps);
  }
  cp_async_wait_all();
  mbar_wait_ab(&sm.xbar, xuse & 1u, err, ab);
  ++xuse;
  named_bar(kBarCons, kCons);

  for (int m = 0; m < M; ++m) {
    const int mode = sm.rmode[m];
    if (mode != HM_SRC_RMS && mode != HM_SRC_EMB) continue;
    uint8_t* xr = xsm + m * xp;
    if (mode == HM_SRC_RMS) {
      const float inv = sm.inv[m];
      const __half* gs = gam_s + sm.rsel[m] * kspan;
      for (int c = tid; c < cpr && 8 * c < K; c += kCons) {
        uint4* slot = reinterpret_cast<uint4*>(xr + c * 16);
        uint4 v = *slot;
        const uint4 gv = *reinterpret_cast<const uint4*>(gs + 8 * c);
        __half2* vh = reinterpret_cast<__half2*>(&v);
        const __half2* gh = reinterpret_cast<const __half2*>(&gv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(vh[j]);
          vh[j] = __hmul2(__floats2half2_rn(f.x * inv, f.y * inv), gh[j]);
        }
        *slot = v;
      }
    } else {
      const float sc = sm.esc[m];
      for (int c = tid; c < cpr && 8 * c < K; c += kCons) {
        uint4* slot = reinterpret_cast<uint4*>(xr + c * 16);
        const uint2 q = *reinterpret_cast<const uint2*>(slot);
        const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
        uint4 v;
        __half* vh = reinterpret_cast<__half*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) vh[j] = __float2half_rn(static_cast<float>(qb[j]) * sc);
        *slot = v;
      }
    }
  }
  named_bar(kBarCons, kCons);

  const __half* const scales = reinterpret_cast<const __half*>(d.s);
  __half* const yout = reinterpret_cast<__half*>(d.y);
  const int64_t ldy = d.ldy, ldres = d.ldres, ss_ld = d.ss_out_ld;
  const __half* const resid = reinterpret_cast<const __half*>(d.res);
  float* const ss_out = d.ss_out;

  const int g = lane >> 2, t = lane & 3;
  const int rot = t >> 1;
  // warp w: box w & 3 of every stage (row block box % rt, k slice box / rt), k-steps 4h .. 4h+3
  const int box = warp & 3, h = warp >> 2;
  const int ksub = box / rt;
  const int er = tid & 15, em0 = tid >> 4;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int n0 = tile * kTileRows + er;
    const int n1 = (rt == 2 ? N / 2 : 0) + tile * kTileRows + er;
    const float sc0 = n0 < N ? __half2float(scales[n0]) : 0.f;
    const float sc1 = (rt == 2 && n1 < N) ? __half2float(scales[n1]) : 0.f;
    // two accumulation chains (even / odd k-steps) keep two MMAs in flight per warp
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int j = 0; j < per_tile; ++j, ++it) {
      const int slot = it % kRing;
      mbar_wait_ab(&sm.full[slot], (it / kRing) & 1, err, ab);
      const uint8_t* wb = sm.ring[slot] + box * kBoxBytes;
      const int wch = ((2 * t + (h ? 1 - rot : rot)) ^ g) << 4;  // this half's 16 weight bytes of the lane
      const uint4 lo = *reinterpret_cast<const uint4*>(wb + g * kBox + wch);
      const uint4 hi = *reinterpret_cast<const uint4*>(wb + (g + 8) * kBox + wch);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
      const uint32_t wa[4] = {lo.x, lo.y, lo.z, lo.w};
      const uint32_t wc[4] = {hi.x, hi.y, hi.z, hi.w};
      const int cb = (j * ks + ksub * kBox) / 8;
      uint32_t xw[8];
      const uint8_t* xr = xsm + g * xp;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + (cb + 4 * t + ((2 * h + i + 2 * rot) & 3)) * 16);
        xw[4 * i + 0] = v.x;
        xw[4 * i + 1] = v.y;
        xw[4 * i + 2] = v.z;
        xw[4 * i + 3] = v.w;
      }
#pragma unroll
      for (int s2 = 0; s2 < 4; ++s2) {
        uint32_t a0, a1, a2, a3;
        i8x4_to_h2x2(wa[s2], a0, a2);
        i8x4_to_h2x2(wc[s2], a1, a3);
        mma_16816(acc[s2 & 1], a0, a1, a2, a3, xw[2 * s2], xw[2 * s2 + 1]);
      }
    }
    float* rw = sm.red + warp * kTileRows * kMP;
    {
      const int m = 2 * t;
      rw[g * kMP + m] = acc[0][0] + acc[1][0];
      rw[g * kMP + m + 1] = acc[0][1] + acc[1][1];
      rw[(g + 8) * kMP + m] = acc[0][2] + acc[1][2];
      rw[(g + 8) * kMP + m + 1] = acc[0][3] + acc[1][3];
    }
    named_bar(kBarCons, kCons);
    // value of (row block b, row r, activation row m): the warps of row block b, in order
    auto value = [&](int b, int r, int m) {
      float a = 0.f;
      for (int w = b; w < kCW; w += rt) a += sm.red[(w * kTileRows + r) * kMP + m];
      return a;
    };
    // epilogue: threads 0..127 (warps 0-3), thread -> (row er of the tile, activation row em0)
    const int m = em0;
    if (warp >= 4) {
      // warps 4-7 have no epilogue share
    } else if (epi == HM_EPI_STORE) {
      float sq = 0.f;
      if (m < M && n0 < N) {
        __half v = __float2half_rn(value(0, er, m) * sc0);
        if (resid) v = hadd_rn(v, resid[(int64_t)m * ldres + n0]);
        yout[(int64_t)m * ldy + n0] = v;
        const float vf = __half2float(v);
        sq = vf * vf;
      }
      if (ss_out) {
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (er == 0 && m < M) ss_out[(int64_t)tile * ss_ld + m] = sq;
      }
    } else if (epi == HM_EPI_ROPE_KV) {
      const int hd = d.hd, qw = d.Hq * d.hd, kw = d.Hk * d.hd;
      const float sc_next = __shfl_down_sync(0xffffffffu, sc0, 1);
      if (!(er & 1) && m < M && n0 < N) {
        const float x0 = __half2float(__float2half_rn(value(0, er, m) * sc0));
        const float x1 = __half2float(__float2half_rn(value(0, er + 1, m) * sc_next));
        const int64_t p = d.pos[m];
        const int bb = m / d.S;
        if (p < 0 || p >= d.L || p >= d.rope_rows) {
          report_error(err, HM_ERR_BADINDEX);
        } else {
          const int dh = n0 % hd;
          __half* kc = reinterpret_cast<__half*>(d.kc);
          __half* vc = reinterpret_cast<__half*>(d.vc);
          if (n0 < qw + kw) {
            const float* cs = d.rope + (p * (hd / 2) + dh / 2) * 2;
            const float c = cs[0], sn = cs[1];
            const __half y0 = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
            const __half y1 = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
            __half* dst;
            if (n0 < qw) {
              dst = reinterpret_cast<__half*>(d.q_out) + (int64_t)m * qw + n0;
            } else {
              const int kh = (n0 - qw) / hd;
              dst = kc + (((int64_t)bb * d.Hk + kh) * d.L + p) * hd + dh;
            }
            dst[0] = y0;
            dst[1] = y1;
          } else {
            const int kh = (n0 - qw - kw) / hd;
            __half* dst = vc + (((int64_t)bb * d.Hk + kh) * d.L + p) * hd + dh;
            dst[0] = __float2half_rn(x0);
            dst[1] = __float2half_rn(x1);
          }
        }
      }
    } else {  // SiLU: row block 0 = w1, row block 1 = w3
      if (m < M) {
        const __half a = __float2half_rn(value(0, er, m) * sc0);
        const __half bv = __float2half_rn(value(1, er, m) * sc1);
        const float af = __half2float(a);
        const __half sl = __float2half_rn(__fdiv_rn(af, __fadd_rn(1.0f, expf(-af))));
        yout[(int64_t)m * ldy + n0] = hmul_rn(sl, bv);
      }
    }
    named_bar(kBarCons, kCons);  // red is reused by the next tile
  }
}

// ---------------------------------------------------------------- attention stage (head_dim 128)
// The 8 consumer warps form two groups of 4; each group runs its own units
// (split, KV head, row) with its own K/V buffers and named barrier.
__device__ void attn_stage(const Stage* st, Smem& sm, uint32_t& atc, int* err) {
  constexpr int HD = 128;
  const AttnStage& A = st->u.a;
  const int gi = threadIdx.x >> 7;               // group
  const int tid = threadIdx.x & 127;             // thread within the group
  const int warp = tid >> 5, lane = tid & 31;    // warp within the group
  const int gbar = 2 + gi;
  TcSmem& ts = *reinterpret_cast<TcSmem*>(sm.xr + gi * kTcBytes);
  uint64_t* abar = sm.abar[gi];
  const CUtensorMap* kmap = &st->map0;
  const CUtensorMap* vmap = &st->map1;
  const int g = lane >> 2, t = lane & 3;
  volatile int* ab = &sm.abort_local;
  const int Hq = A.Hq, Hk = A.Hk, S = A.S, L = A.L, nsplit = A.nsplit, R = A.R;
  const int G = Hq / Hk;
  const float scale = A.scale;
  const int units = nsplit * Hk * R;
  if (tid == 0) {
    prefetch_tensormap(kmap);
    prefetch_tensormap(vmap);
  }
  const int mi = lane >> 3, ri = lane & 7;
  for (int u = 2 * blockIdx.x + gi; u < units; u += 2 * gridDim.x) {
    const int sp = u % nsplit, kh = (u / nsplit) % Hk, r = u / (nsplit * Hk);
    const int64_t p_last = A.pos[r];
    const int b = r / S;
    int len = static_cast<int>(p_last) + 1;
    if (p_last < 0 || p_last >= L) {
      if (tid == 0) report_error(err, HM_ERR_BADINDEX);
      len = 0;
    }
    const int per = (len + nsplit - 1) / nsplit;
    const int chunk = (per + kTcPos - 1) / kTcPos * kTcPos;
    const int lo = sp * chunk;
    const int hi = min(len, lo + chunk);
    const int ntile = hi > lo ? (hi - lo + kTcPos - 1) / kTcPos : 0;
    const int row0 = ((b * Hk + kh) * L) + lo;
    const uint32_t atc0 = atc;
    auto issue = [&](int tt) {
      const int stg = (atc0 + tt) % kTcNst;
      const int y = row0 + tt * kTcPos;
      mbar_arrive_expect_tx(&abar[stg], 4 * kTcBox);
      tma_load_2d_plain(ts.k[stg][0], kmap, 0, y, &abar[stg]);
      tma_load_2d_plain(ts.k[stg][1], kmap, 64, y, &abar[stg]);
      tma_load_2d_plain(ts.v[stg][0], vmap, 0, y, &abar[stg]);
      tma_load_2d_plain(ts.v[stg][1], vmap, 64, y, &abar[stg]);
    };
    if (tid == 0)
      for (int tt = 0; tt < kTcNst && tt < ntile; ++tt) issue(tt);

    uint32_t qa[8][2];
    {
      const __half* qh = A.q + ((int64_t)r * Hq + kh * G + g) * HD;
#pragma unroll
      for (int k2 = 0; k2 < 8; ++k2) {
        qa[k2][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + 16 * k2 + 2 * t) : 0u;
        qa[k2][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + 16 * k2 + 8 + 2 * t) : 0u;
      }
    }
    float m_run = -INFINITY, l_run = 0.f;
    float acc[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (int tt = 0; tt < ntile; ++tt) {
      const uint32_t n_use = atc0 + tt;
      const int stg = n_use % kTcNst;
      mbar_wait_ab(&abar[stg], (n_use / kTcNst) & 1, err, ab);
      const int nvalid = min(16, hi - (lo + tt * kTcPos + warp * 16));
      if (nvalid > 0) {
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int kp = warp * 16 + (mi >= 2 ? 8 : 0) + ri;
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2) {
          const int c = 2 * k2 + (mi & 1);
          uint32_t b00, b01, b10, b11;
          ldsm_x4(b00, b01, b10, b11, swz(ts.k[stg][c >> 3], kp, c & 7));
          mma_16816(s[0], qa[k2][0], 0u, qa[k2][1], 0u, b00, b01);
          mma_16816(s[1], qa[k2][0], 0u, qa[k2][1], 0u, b10, b11);
        }
        float v4[4];
        float tmax = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int pl = 8 * n + 2 * t + e;
            const float val = pl < nvalid ? s[n][e] * scale : -INFINITY;
            v4[2 * n + e] = val;
            tmax = fmaxf(tmax, val);
          }
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float m_new = fmaxf(m_run, tmax);
        float alpha = 1.f, psum = 0.f;
        float pv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pv[i] = (m_new == -INFINITY || v4[i] == -INFINITY) ? 0.f : expf(v4[i] - m_new);
          psum += pv[i];
        }
        if (m_new != -INFINITY) alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        l_run = l_run * alpha + psum;
        m_run = m_new;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          acc[i][0] *= alpha;
          acc[i][1] *= alpha;
        }
        const uint32_t pa0 = pack_h2(pv[0], pv[1]), pa2 = pack_h2(pv[2], pv[3]);
        const int vp = warp * 16 + (mi & 1) * 8 + ri;
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
          const int c = 2 * nd + (mi >> 1);
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(v0, v1, v2, v3, swz(ts.v[stg][c >> 3], vp, c & 7));
          mma_16816(acc[2 * nd], pa0, 0u, pa2, 0u, v0, v1);
          mma_16816(acc[2 * nd + 1], pa0, 0u, pa2, 0u, v2, v3);
        }
      }
      named_bar(gbar, 128);  // every warp is done with this buffer
      if (tid == 0 && tt + kTcNst < ntile) issue(tt + kTcNst);
    }
    atc = atc0 + ntile;

    // ---- merge the four warps (red aliases stage-0 K of the next unit: all loads consumed)
    float* red = reinterpret_cast<float*>(&ts.k[0][0][0]);  // [4][kMaxG][128]
    if (g < G) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        red[(warp * kMaxG + g) * HD + 8 * i + 2 * t] = acc[i][0];
        red[(warp * kMaxG + g) * HD + 8 * i + 2 * t + 1] = acc[i][1];
      }
      if (t == 0) {
        ts.mw[warp][g] = m_run;
        ts.lw[warp][g] = l_run;
      }
    }
    named_bar(gbar, 128);
    const int64_t head0 = (int64_t)r * Hq + kh * G;
    const int64_t nh = (int64_t)R * Hq * nsplit;
    float* wm = A.ws;
    float* wl = A.ws + nh;
    float* wa = A.ws + 2 * nh;
    for (int i = tid; i < G * HD; i += 128) {
      const int gg = i / HD, dd = i - gg * HD;
      float Mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) Mx = fmaxf(Mx, ts.mw[w][gg]);
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float mw = ts.mw[w][gg];
        const float f = mw > -INFINITY ? expf(mw - Mx) : 0.f;
        num += red[(w * kMaxG + gg) * HD + dd] * f;
        den += ts.lw[w][gg] * f;
      }
      if (nsplit == 1) {
        A.o[(head0 + gg) * HD + dd] = __float2half_rn(den > 0.f ? num / den : 0.f);
      } else {
        wa[((head0 + gg) * nsplit + sp) * HD + dd] = num;
        if (dd == 0) {
          wm[(head0 + gg) * nsplit + sp] = Mx;
          wl[(head0 + gg) * nsplit + sp] = den;
        }
      }
    }
    if (nsplit > 1) {
      __threadfence();
      named_bar(gbar, 128);
      int* ticket = &A.counters[r * Hk + kh];
      if (tid == 0) ts.flag = (atomicAdd(ticket, 1) == nsplit - 1);
      named_bar(gbar, 128);
      if (ts.flag) {
        __threadfence();
        for (int i = tid; i < G * nsplit; i += 128) {
          const int gg = i / nsplit, s2 = i - gg * nsplit;
          ts.cw[gg][s2] = __ldcg(wm + (head0 + gg) * nsplit + s2);
          ts.cl[gg][s2] = __ldcg(wl + (head0 + gg) * nsplit + s2);
        }
        named_bar(gbar, 128);
        if (tid < G) {
          float mx = -INFINITY;
          for (int s2 = 0; s2 < nsplit; ++s2) mx = fmaxf(mx, ts.cw[tid][s2]);
          float den = 0.f;
          for (int s2 = 0; s2 < nsplit; ++s2) {
            const float ms = ts.cw[tid][s2];
            const float w = ms > -INFINITY ? expf(ms - mx) : 0.f;
            ts.cw[tid][s2] = w;
            den += ts.cl[tid][s2] * w;
          }
          ts.cden[tid] = den;
        }
        named_bar(gbar, 128);
        for (int i = tid; i < G * HD; i += 128) {
          const int gg = i / HD, dd = i - gg * HD;
          const int64_t h = head0 + gg;
          float num = 0.f;
          for (int s2 = 0; s2 < nsplit; ++s2) num += __ldcg(wa + (h * nsplit + s2) * HD + dd) * ts.cw[gg][s2];
          const float den = ts.cden[gg];
          A.o[h * HD + dd] = __float2half_rn(den > 0.f ? num / den : 0.f);
        }
        if (tid == 0) *ticket = 0;
      }
    }
    fence_proxy_async_smem();    // generic writes above before the next unit's TMA writes
    named_bar(gbar, 128);  // the buffers are reused by the next unit
  }
}

// ---------------------------------------------------------------- embedding sum stage
// x[r, k] = fp16( sum_c fp16(q8[tok[r,c] + c*V, k] * s8[...]) ) and per-16-column sums of squares
__device__ void embsum_stage(const Stage* st, int* err) {
  constexpr int kMaxCb = 16;
  const EmbStage& E = st->u.e;
  const int tid = threadIdx.x;
  const int D = E.D, ncb = E.ncb;
  const int per_row = (D + kCons - 1) / kCons;
  for (int u = blockIdx.x; u < E.R * per_row; u += gridDim.x) {
    const int r = u / per_row, k = (u % per_row) * kCons + tid;
    // all codebook rows' bytes in flight together, then the sum in codebook order
    int8_t q[kMaxCb];
    float sc[kMaxCb];
#pragma unroll
    for (int c = 0; c < kMaxCb; ++c) {
      q[c] = 0;
      sc[c] = 0.f;
      if (c < ncb && k < D) {
        const int64_t id = E.tok[(int64_t)r * E.tok_ld + c] + c * E.vocab;
        if (id < 0 || id >= E.rows) {
          report_error(err, HM_ERR_BADINDEX);
        } else {
          q[c] = E.tab[id * D + k];
          sc[c] = __half2float(E.scale[id]);
        }
      }
    }
    float a = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxCb; ++c)
      if (c < ncb) a += __half2float(__float2half_rn(static_cast<float>(q[c]) * sc[c]));
    const __half v = __float2half_rn(a);
    if (k < D) E.x[(int64_t)r * D + k] = v;
    if (E.ss) {
      float sq = k < D ? __half2float(v) * __half2float(v) : 0.f;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if ((tid & 15) == 0 && k < D) E.ss[(int64_t)(k / 16) * E.ss_ld + r] = sq;
    }
  }
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 1) seq_kernel(const __grid_constant__ SeqCtl C) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    sm.abort_local = 0;
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kCW);
    }
    mbar_init(&sm.xbar, 1);
    for (int i = 0; i < kTcNst; ++i) {
      mbar_init(&sm.abar[0][i], 1);
      mbar_init(&sm.abar[1][i], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const SeqCtl c = C;
  if (warp == kCW) {
    if ((tid & 31) == 0) producer(c, sm);
    return;
  }
  int it = 0;
  uint32_t xuse = 0, atc = 0;
  for (int s = 0; s < c.n; ++s) {
    if (s > 0) grid_wait(c, static_cast<unsigned>(s) * gridDim.x, tid);
    const Stage* st = c.stages + s;
    const int type = st->type;
    if (type == ST_GEMV) gemv_stage(st, sm, it, xuse, c.err);
    else if (type == ST_ATTN) attn_stage(st, sm, atc, c.err);
    else embsum_stage(st, c.err);
    grid_arrive(c, tid);
  }
}

int sm_count_of_current() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// ---------------------------------------------------------------- C ABI
struct hm_seq {
  std::vector<Stage> stages;
  Stage* d_stages = nullptr;
  unsigned* d_ctl = nullptr;  // [0] barrier counter, [1] abort flag
  int uploaded = 0;
  int grid = 0;
};

extern "C" hm_seq* hm_seq_create(void) { return new (std::nothrow) hm_seq(); }

extern "C" void hm_seq_destroy(hm_seq* q) {
  if (!q) return;
  if (q->d_stages) cudaFree(q->d_stages);
  if (q->d_ctl) cudaFree(q->d_ctl);
  delete q;
}

extern "C" int hm_seq_size(const hm_seq* q) { return q ? static_cast<int>(q->stages.size()) : 0; }

bool hm_seq_weight_map(const int8_t* w, int N, int K, CUtensorMap* out);  // gemv_i8.cu
bool hm_seq_cache_map(const void* base, int64_t rows, CUtensorMap* out);  // decode_attn.cu

extern "C" int hm_seq_add_gemv(hm_seq* q, const hm_gemv_desc* d, int keep) {
  if (!q || q->uploaded || !d || !d->w || !d->s || d->M < 1 || d->M > kRows || d->N < 1 || d->K < 16 ||
      d->K % 16 || !aligned16(d->w))
    return HM_EARG;
  if (d->epi == HM_EPI_SILU && (d->N % (2 * kTileRows) || !d->y)) return HM_EARG;
  if (d->epi == HM_EPI_STORE && (!d->y || (d->ss_out && d->N % kTileRows))) return HM_EARG;
  if (d->epi == HM_EPI_ROPE_KV &&
      (!d->rope || !d->pos || !d->q_out || !d->kc || !d->vc || d->hd % kTileRows || d->S < 1 ||
       d->N != (d->Hq + 2 * d->Hk) * d->hd))
    return HM_EARG;
  if (d->epi != HM_EPI_STORE && d->epi != HM_EPI_ROPE_KV && d->epi != HM_EPI_SILU) return HM_EARG;
  int has_gamma = 0;
  for (int i = 0; i < (d->interleave ? 2 : 1); ++i) {
    const hm_row_src& s = d->src[i];
    if (s.mode == HM_SRC_EMB) {
      if (!s.etab || !s.escale || !s.tok || (reinterpret_cast<uintptr_t>(s.etab) & 7u) || d->K % 8) return HM_EARG;
    } else if (s.mode == HM_SRC_F16 || s.mode == HM_SRC_RMS) {
      if (!s.x || !aligned16(s.x) || (s.ldx % 8)) return HM_EARG;
      if (s.mode == HM_SRC_RMS) {
        if (!s.ss || !s.gamma || !aligned16(s.gamma) || s.dim <= 0) return HM_EARG;
        has_gamma = 1;
      }
    } else {
      return HM_EARG;
    }
  }
  Stage st;
  memset(&st, 0, sizeof(st));
  st.type = ST_GEMV;
  GemvStage& g = st.u.g;
  g.d = *d;
  g.rt = d->epi == HM_EPI_SILU ? 2 : 1;
  g.ks = 4 * kBox / g.rt;
  g.kspan = (d->K + g.ks - 1) / g.ks * g.ks;
  g.per_tile = g.kspan / g.ks;
  g.ntiles = d->epi == HM_EPI_SILU ? (d->N / 2) / kTileRows : (d->N + kTileRows - 1) / kTileRows;
  g.has_gamma = has_gamma;
  g.keep = keep ? 1 : 0;
  const int xbytes = kRows * (g.kspan * 2 + 16) + (has_gamma ? 2 * g.kspan * 2 : 0);
  if (xbytes > kXRegion) return HM_ENOSPACE;
  if (!hm_seq_weight_map(d->w, d->N, d->K, &st.map0)) return HM_EARG;
  q->stages.push_back(st);
  return HM_OK;
}

extern "C" int hm_seq_add_attn(hm_seq* q, const void* qv, const void* kc, const void* vc, const int64_t* pos, void* o,
                               int R, int S, int Hq, int Hk, int hd, int L, float scale, int nsplit, void* ws,
                               size_t ws_bytes, int* counters, int n_counters) {
  if (!q || q->uploaded || !qv || !kc || !vc || !pos || !o || R < 1 || S < 1 || R % S || Hk < 1 || Hq % Hk ||
      hd != 128 || L < 1 || nsplit < 1 || nsplit > kMaxSplit || Hq / Hk > kMaxG)
    return HM_EARG;
  if (nsplit > 1) {
    const size_t need = static_cast<size_t>(R) * Hq * nsplit * (hd + 2) * sizeof(float);
    if (!ws || ws_bytes < need || !counters || n_counters < R * Hk) return HM_EARG;
  }
  Stage st;
  memset(&st, 0, sizeof(st));
  st.type = ST_ATTN;
  AttnStage& a = st.u.a;
  a.q = reinterpret_cast<const __half*>(qv);
  a.pos = pos;
  a.o = reinterpret_cast<__half*>(o);
  a.R = R;
  a.S = S;
  a.Hq = Hq;
  a.Hk = Hk;
  a.L = L;
  a.nsplit = nsplit;
  a.scale = scale;
  a.ws = reinterpret_cast<float*>(ws);
  a.counters = counters;
  const int64_t rows = static_cast<int64_t>(R / S) * Hk * L;
  if (!hm_seq_cache_map(kc, rows, &st.map0) || !hm_seq_cache_map(vc, rows, &st.map1)) return HM_EARG;
  q->stages.push_back(st);
  return HM_OK;
}

extern "C" int hm_seq_add_emb_sum(hm_seq* q, const int64_t* tok, int64_t tok_ld, int R, int ncb, int64_t vocab,
                                  const int8_t* tab, const void* scale, int64_t rows, int D, void* x_out,
                                  float* ss_out, int64_t ss_ld) {
  if (!q || q->uploaded || !tok || !tab || !scale || !x_out || R < 1 || ncb < 1 || ncb > 16 || D < 1 || D % 16)
    return HM_EARG;
  Stage st;
  memset(&st, 0, sizeof(st));
  st.type = ST_EMBSUM;
  EmbStage& e = st.u.e;
  e.tok = tok;
  e.tok_ld = tok_ld;
  e.ncb = ncb;
  e.vocab = vocab;
  e.tab = tab;
  e.scale = reinterpret_cast<const __half*>(scale);
  e.rows = rows;
  e.R = R;
  e.D = D;
  e.x = reinterpret_cast<__half*>(x_out);
  e.ss = ss_out;
  e.ss_ld = ss_ld;
  q->stages.push_back(st);
  return HM_OK;
}

// Upload the stage list (allocates the descriptor array once; call outside stream capture).
extern "C" int hm_seq_finalize(hm_seq* q) {
  if (!q || q->stages.empty()) return HM_EARG;
  if (q->uploaded) return HM_OK;
  const size_t bytes = q->stages.size() * sizeof(Stage);
  cudaError_t e = cudaMalloc(&q->d_stages, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMalloc(&q->d_ctl, 64);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemcpy(q->d_stages, q->stages.data(), bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(q->d_ctl, 0, 64);
  if (e != cudaSuccess) return static_cast<int>(e);
  const size_t smem = sizeof(Smem) + 1024;
  e = cudaFuncSetAttribute(seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, seq_kernel, kThreads, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (occ < 1) return HM_EARG;
  q->grid = sm_count_of_current();  // one CTA per SM (the shared memory allows no second)
  q->uploaded = 1;
  return HM_OK;
}

// Launch the sequence on `stream` (capturable): zero the barrier, then one cooperative launch.
extern "C" int hm_seq_launch(hm_seq* q, int* err, hm_stream_t stream) {
  if (!q || !q->uploaded) return HM_EARG;
  cudaError_t e = cudaMemsetAsync(q->d_ctl, 0, 8, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  SeqCtl c;
  c.stages = q->d_stages;
  c.n = static_cast<int>(q->stages.size());
  c.barrier = q->d_ctl;
  c.abort = reinterpret_cast<int*>(q->d_ctl + 1);
  c.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(q->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(Smem) + 1024;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, seq_kernel, c);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" size_t hm_seq_smem_bytes(void) { return sizeof(Smem) + 1024; }
