// int8 weight-only GEMV / skinny GEMM for the HeartMuLa decode path (sm_100a).
//
// Replaces the reference's `_gemv8` Triton kernel and its `int8_mm` dispatcher
// (app/kernels.py:20-54) and fuses what surrounds it in Stack.decode
// (app/engine.py:180-211): RMSNorm or an int8 embedding gather in the
// prologue; residual add, RoPE + KV-cache write, or SiLU*mul in the epilogue.
//
// Design (HBM-bound: every weight byte is read exactly once per frame):
//  * Tiles of 16 weight rows (16 w1 + 16 w3 rows for the SiLU epilogue) over a
//    k-range that is the whole K whenever the activations fit in shared memory
//    (every decode shape at up to 8 rows), so no cross-CTA reduction is needed.
//    One wave of persistent CTAs strides over the tiles.
//  * A producer warp streams each tile through a 6-stage ring of 8 KB stages
//    (four 16x128-byte TMA boxes, 128B swizzle, L2 evict-first), running ahead
//    across tile boundaries and starting before griddepcontrol.wait, so the
//    weight stream of a launch overlaps the tail of the previous launch.
//  * Four consumer warps stage the activation k-range once per CTA (all loads
//    in flight together: cp.async for fp16 rows, ids then int8 rows for
//    embedding gathers, RMSNorm applied in place); each warp takes one of the
//    stage's four boxes (a 128-column slice) and runs tensor-core MMA m16n8k16
//    with the weights as the 16-row A operand and up to 8*MT activation rows as
//    the n dimension ("swap AB": at R = 8 rows there is no padding).  int8 ->
//    fp16 is exact, accumulation is fp32, and the per-row scale is applied
//    afterwards in fp32, where _gemv8 applies it.  The four warps' partial sums
//    are added in a fixed order (deterministic).
//  * K inside a 128-column box is permuted consistently for A and B so every
//    lane reads 32 contiguous weight bytes and 64 contiguous activation bytes.
//  * Only when the activations do not fit (many rows x long K) the k-range is
//    split over CTAs; partials then go to scratch and the last CTA of a tile
//    (atomic ticket) sums them in split order and runs the epilogue.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "hm_common.cuh"

namespace {

constexpr int kTileRows = 16;   // rows of one MMA row block
constexpr int kBox = 128;       // k columns (bytes) per TMA box
constexpr int kBoxBytes = kTileRows * kBox;
constexpr int kStage = 4 * kBoxBytes;  // four boxes per stage
constexpr int kNST = 6;         // ring stages at the default depth
constexpr int kMaxNST = 14;     // deepest ring (the mbarrier arrays are sized for it)
constexpr int kGW = 4;          // MMA warps of one consumer group (one box of a stage each)
constexpr int kGT = 32 * kGW;   // threads of one consumer group
constexpr int kMaxGroups = 4;   // consumer groups of the wide kernel
__host__ __device__ constexpr int threads_of(int groups) { return 32 * (kGW * groups + 1); }
constexpr int kMaxM = 32;
constexpr int kMaxCSplit = 8;   // k-ranges of one tile in a cluster (portable cluster size)
constexpr int kBarCons = 1;     // named barrier of all consumer warps
constexpr int kBarGrp = 2;      // named barriers 2.. : one per consumer group

struct GemvParams {
  hm_gemv_desc d;
  int kspan, nsplit, ntiles;
  int has_gamma;  // gamma vectors staged: 0, 1 (src[0]) or 2 (interleaved sources)
  int xcontig;  // the M input rows are one contiguous block: staged by one bulk copy, unpadded pitch
  int xf_loop;  // every row is RMS(src[0]): CTAs with one tile normalise in registers in the MMA loop
  int nst;      // ring stages: deeper when the CTAs per SM leave shared memory free
  int cluster;  // the nsplit k-ranges of a tile run as one thread-block cluster and reduce in DSMEM
  int groups;   // consumer groups in use (wide kernel): each streams its own tiles through its own ring
  int box;      // weight map: 0 = 2-D, four 16-row x 128-byte boxes per stage; 1 = one box per stage
                // (3-D for one row block, 4-D for the w1|w3 pair: the same shared-memory layout)
};

struct SmemLayout {
  int ring, x, gam, red, cpart, inv, esc, rowp, rmode, flag, bars, total;  // flag: [g] tile owner of group g, [7] abort
  int xp;  // activation row pitch in bytes
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }
__host__ __device__ inline int rt_of(int epi) { return epi == HM_EPI_SILU ? 2 : 1; }
__host__ __device__ inline int ks_of(int epi) { return 4 * kBox / rt_of(epi); }  // k bytes per stage

__host__ __device__ inline SmemLayout smem_layout(int kspan, int mrows, int has_gamma, int xcontig = 0,
                                                  int nst = kNST, int groups = 1) {
  SmemLayout L;
  L.ring = 0;  // one ring of nst stages per consumer group
  L.xp = kspan * 2 + (xcontig ? 0 : 16);
  L.x = groups * nst * kStage;
  L.gam = align_up(L.x + mrows * L.xp, 16);
  L.red = L.gam + has_gamma * kspan * 2;
  L.cpart = L.red + groups * kGW * kTileRows * (mrows + 1) * 4;  // this k-range's partial tile (cluster split)
  L.inv = L.cpart + 2 * kTileRows * mrows * 4;
  L.esc = L.inv + kMaxM * 4;
  L.rowp = align_up(L.esc + kMaxM * 4, 8);
  L.rmode = L.rowp + kMaxM * 8;
  L.flag = L.rmode + 2 * kMaxM * 4;
  L.bars = align_up(L.flag + 32, 8);
  L.total = L.bars + (2 * groups * kMaxNST + 3) * 8;
  return L;
}

// Activation rows are stored linearly (one bulk copy per row) with a pitch of
// 16 mod 128 bytes.  Lane (g, t) reads the four 16-byte chunks 4t..4t+3 of its
// 128-column slice; lanes with t >= 2 read them rotated by two chunks (and take
// the two halves of their weight bytes swapped to match), which keeps the eight
// lanes of every shared-memory phase on distinct banks.

// Named barrier of consumer group `grp` (kGT threads).  The ids are spelled as constants
// so ptxas reserves only the barriers the kernel names (a register id reserves all 16,
// which limits the CTAs per SM).
template <int GR>
__device__ __forceinline__ void group_bar(int grp) {
  if (GR == 1) {
    named_bar(kBarCons, kGT);  // one group: the consumer barrier itself (two barriers per CTA)
  } else {
    switch (grp) {
      case 0: named_bar(kBarGrp, kGT); break;
      case 1: named_bar(kBarGrp + 1, kGT); break;
      case 2: named_bar(kBarGrp + 2, kGT); break;
      default: named_bar(kBarGrp + 3, kGT); break;
    }
  }
}

__device__ __forceinline__ const hm_row_src& src_of(const hm_gemv_desc& d, int m, int& row, int& sel) {
  sel = d.interleave ? (m & 1) : 0;
  const int local = d.interleave ? (m >> 1) : m;
  const hm_row_src& s = d.src[sel];
  row = local * s.row_mul + s.row_add;
  return s;
}


// GR consumer groups of four MMA warps (GR = 1: one group, the split-K and many-row
// shapes; GR = 4: the wide kernel, one CTA per SM).  Each group owns a ring of weight
// stages fed by its own producer lane and streams its own tiles (the CTA's tiles g,
// g + groups, ...), so the tiles of an SM run concurrently; all groups share one
// staging of the activations, which every consumer warp helps to prepare.
// (launch bounds: the narrow 8-row kernel is left to the compiler's register choice -- a
// minimum-blocks bound changed its schedule and measured ~10 % slower at the same
// register count; the wider-row kernels ask for two CTAs per SM, the wide kernel one)
template <int MT, int EPI, int GR>
__global__ void __launch_bounds__(threads_of(GR), GR == 1 ? (MT == 1 ? 0 : 2) : 1) gemv_i8_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                    const __grid_constant__ GemvParams P) {
  constexpr int kCons = kGT * GR;  // consumer threads
  // EPI < 0: one instantiation for every epilogue, read from the parameters (the
  // launches of a layer then share their prologue and MMA-loop code in the SM's
  // instruction cache); EPI >= 0 folds it at compile time
  const int epi = EPI >= 0 ? EPI : P.d.epi;
  const int RT = epi == HM_EPI_SILU ? 2 : 1;
  const int KS = 4 * kBox / RT;
  constexpr int MROWS = 8 * MT;
  constexpr int MP = MROWS + 1;
  extern __shared__ __align__(1024) uint8_t smem[];
  const hm_gemv_desc& d = P.d;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int kspan = P.kspan;
  const int k0 = split * kspan;
  const int M = d.M;
  const int per_tile = kspan / KS;  // stages per tile
  const int my_tiles = (P.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int G = GR == 1 ? 1 : P.groups;  // groups in use (<= GR)
  const int nst = P.nst;
  const SmemLayout L = smem_layout(kspan, MROWS, P.has_gamma, P.xcontig, nst, G);
  uint8_t* ring = smem + L.ring;
  uint8_t* xsm = smem + L.x;
  __half* gam_s = reinterpret_cast<__half*>(smem + L.gam);
  float* red_s = reinterpret_cast<float*>(smem + L.red);
  float* inv_s = reinterpret_cast<float*>(smem + L.inv);
  float* esc_s = reinterpret_cast<float*>(smem + L.esc);
  const uint8_t** rowp_s = reinterpret_cast<const uint8_t**>(smem + L.rowp);
  int* rmode_s = reinterpret_cast<int*>(smem + L.rmode);
  int* rsel_s = rmode_s + kMaxM;
  int* flag_s = reinterpret_cast<int*>(smem + L.flag);
  volatile int* abort_s = flag_s + 7;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [group][kMaxNST]
  uint64_t* empty = full + G * kMaxNST;
  uint64_t* xbar = empty + G * kMaxNST;  // bulk copies of the activation rows and gammas
  uint64_t* cready = xbar + 1;       // cluster split: the other k-ranges' partials are in (rank 0)
  uint64_t* cdone = xbar + 2;        // cluster split: rank 0 has read this CTA's partial
  float* cpart_s = reinterpret_cast<float*>(smem + L.cpart);

  if (smem_u32(ring) & 1023u) {  // 128B-swizzled TMA destinations must be 1024-byte aligned
    if (tid == 0) report_error(d.err, HM_ERR_TIMEOUT);
    return;
  }
  // ring barriers initialised one per thread (one thread takes ~1 us for the ~100 of the
  // wide kernel, on the way to the dependency wait); each thread fences its own
  for (int i = tid; i < G * nst; i += static_cast<int>(blockDim.x)) {
    mbar_init(&full[(i / nst) * kMaxNST + i % nst], 1);
    mbar_init(&empty[(i / nst) * kMaxNST + i % nst], kGW);
  }
  if (tid == 0) {
    *abort_s = 0;
    mbar_init(xbar, 1);
    if (P.cluster) {
      mbar_init(cready, P.nsplit - 1);
      mbar_init(cdone, 1);
    }
  }
  fence_barrier_init();
  __syncthreads();
  if (P.cluster) cluster_sync_all();  // every CTA's split barriers exist before any remote arrival

  // ================================================================ producer warp
  if (warp == kCons / 32) {
    pdl_trigger();
    if (lane < G) {  // lane g feeds group g's ring with the stages of the group's tiles
      const int g = lane;
      int* const perr = d.err;
      const int half_n = d.N / 2;
      if (g == 0) prefetch_tensormap(&wmap);
      const uint64_t pol = d.l2_keep ? policy_evict_last() : policy_evict_first();
      const int tiles_g = my_tiles > g ? (my_tiles - g + G - 1) / G : 0;
      const int nstages = tiles_g * per_tile;
      uint8_t* const gring = ring + g * nst * kStage;
      uint64_t* const gfull = full + g * kMaxNST;
      uint64_t* const gempty = empty + g * kMaxNST;
      int slot = 0, round = 0;  // it = round * nst + slot
      for (int it = 0; it < nstages; ++it) {
        if (round > 0) mbar_wait_ab(&gempty[slot], (round - 1) & 1, perr, abort_s);
        const int tile = (int)blockIdx.x + (g + (it / per_tile) * G) * (int)gridDim.x;
        const int kx = k0 + (it % per_tile) * KS;
        mbar_arrive_expect_tx(&gfull[slot], kStage);
        if (P.box) {  // one request per stage (the TMA unit's cost is per box as much as per byte)
          if (RT == 1)
            tma_load_3d(gring + slot * kStage, &wmap, 0, tile * kTileRows, kx / kBox, &gfull[slot], pol);
          else
            tma_load_4d(gring + slot * kStage, &wmap, 0, tile * kTileRows, 0, kx / kBox, &gfull[slot], pol);
        } else {
#pragma unroll
          for (int b = 0; b < 4; ++b)
            tma_load_2d(gring + slot * kStage + b * kBoxBytes, &wmap, kx + (b / RT) * kBox,
                        (RT == 2 && (b % RT) == 1 ? half_n : 0) + tile * kTileRows, &gfull[slot], pol);
        }
        if (++slot == nst) {
          slot = 0;
          ++round;
        }
      }
    }
    pdl_wait();
    return;
  }

  // ================================================================ consumer warps
  pdl_trigger();

  // Before griddepcontrol.wait: everything that depends only on the launch parameters
  // and immutable data (row pointers of fp16 / RMS rows, the gamma copies, zeros for
  // padding rows and tails), so the dependent part starts with the activation copy.
  //
  // Parameter fields are copied to registers / shared memory once: the inline-asm
  // copies and barriers below clobber memory, which would otherwise force a reload
  // of every field through the parameter block on each loop iteration.
  const int K = d.K, N = d.N;
  int* const err = d.err;

  // ---- per-row sources: mode and source index; row pointers of fp16 / RMS rows
  // (embedding rows need their token ids, which earlier launches write)
  if (tid < MROWS) {
    const int m = tid;
    int mode = -1;  // -1: padding row or rejected id -> zeros
    int sel = 0;
    const uint8_t* base = nullptr;
    if (m < M) {
      int row;
      const hm_row_src& s = src_of(d, m, row, sel);
      mode = s.mode;
      if (mode != HM_SRC_EMB)
        base = reinterpret_cast<const uint8_t*>(reinterpret_cast<const __half*>(s.x) + (int64_t)row * s.ldx);
    }
    rmode_s[m] = mode;
    rsel_s[m] = sel;
    rowp_s[m] = base;
    esc_s[m] = 0.f;
  }
  const __half* gam0 = reinterpret_cast<const __half*>(d.src[0].gamma);
  const __half* gam1 = reinterpret_cast<const __half*>(d.src[1].gamma);
  const bool g0 = P.has_gamma && d.src[0].mode == HM_SRC_RMS;
  const bool g1 = P.has_gamma && d.interleave && d.src[1].mode == HM_SRC_RMS;
  named_bar(kBarCons, kCons);

  // ---- stage the activation k-range [MROWS][kspan]: one bulk copy per fp16 / RMS row
  // and per gamma (thread 0), 8-byte cp.async for int8 embedding rows (into the first
  // half of each 16-byte chunk), zeros for padding rows, rejected ids and the tail
  const int cpr = kspan / 8;
  const int kend = min(kspan, K - k0);  // valid columns of this k-range (a multiple of 8)
  bool any_emb = false;
  for (int m = 0; m < M; ++m) any_emb |= rmode_s[m] == HM_SRC_EMB;
  if (tid == 0) {  // expected bytes of the whole staging; the gammas are weights: issued now
    uint32_t bytes = 0;
    for (int m = 0; m < M; ++m) bytes += (rmode_s[m] == HM_SRC_F16 || rmode_s[m] == HM_SRC_RMS) ? kend * 2 : 0;
    bytes += (g0 ? kend * 2 : 0) + (g1 ? kend * 2 : 0);
    mbar_arrive_expect_tx(xbar, bytes);
    if (g0) bulk_load(gam_s, gam0 + k0, kend * 2, xbar);
    if (g1) bulk_load(gam_s + kspan, gam1 + k0, kend * 2, xbar);
  }
  // (row-uniform branches: fp16/RMS/embedding rows only need their tail zeroed, usually none)
  const int ctail = kend / 8;  // first chunk past the valid columns
  for (int m = 0; m < MROWS; ++m) {
    const int mode = m < M ? rmode_s[m] : -1;
    uint8_t* xr = xsm + m * L.xp;
    for (int c = (mode < 0 ? 0 : ctail) + tid; c < cpr; c += kCons)
      *reinterpret_cast<uint4*>(xr + c * 16) = make_uint4(0, 0, 0, 0);
  }
  // RMSNorm in the MMA loop (registers) instead of a shared-memory pass: in CTAs with one
  // tile (the pass and the loop then touch each element once either way, the loop without
  // a barrier and a store) and one row block per stage (with two, two warps would
  // normalise the same columns)
  const bool xf_loop = P.xf_loop && RT == 1 && my_tiles <= G;
  if (xf_loop)  // gamma past K meets zero activations in the MMA loop: keep it finite
    for (int c = ctail + tid; c < cpr; c += kCons) reinterpret_cast<uint4*>(gam_s)[c] = make_uint4(0, 0, 0, 0);

  // epilogue parameters, in registers for the whole tile loop (read before the wait:
  // the first touch of a parameter field misses the constant cache)
  const __half* const scales = reinterpret_cast<const __half*>(d.s);
  __half* const yout = reinterpret_cast<__half*>(d.y);
  const int64_t ldy = d.ldy, ldres = d.ldres, ss_ld = d.ss_out_ld;
  const __half* const resid = reinterpret_cast<const __half*>(d.res);
  float* const ss_out = d.ss_out;
  float* const wsp = reinterpret_cast<float*>(d.ws);
  int* const counters = d.counters;
  struct RopeP {
    int hd, qw, kw, S, L, Hk, rope_rows;
    const int64_t* pos;
    const float* rope;
    __half *qo, *kc, *vc;
  } rp{};
  if (epi == HM_EPI_ROPE_KV) {
    rp.hd = d.hd;
    rp.qw = d.Hq * d.hd;
    rp.kw = d.Hk * d.hd;
    rp.S = d.S;
    rp.L = d.L;
    rp.Hk = d.Hk;
    rp.rope_rows = d.rope_rows;
    rp.pos = d.pos;
    rp.rope = d.rope;
    rp.qo = reinterpret_cast<__half*>(d.q_out);
    rp.kc = reinterpret_cast<__half*>(d.kc);
    rp.vc = reinterpret_cast<__half*>(d.vc);
  }

  // consumer group of this warp and the group's tiles (the CTA's tiles grp, grp + G, ...)
  const int grp = GR == 1 ? 0 : warp / kGW, gw = GR == 1 ? warp : warp % kGW, gtid = GR == 1 ? tid : tid % kGT;
  const int tiles_g = grp < G && my_tiles > grp ? (my_tiles - grp + G - 1) / G : 0;
  // per-row weight scales of this thread's epilogue rows (immutable): the group's first
  // tile's now, each next tile's while the current one streams
  const int er = gtid & 15, em0 = gtid >> 4;
  const int half_n = RT == 2 ? N / 2 : 0;
  int nn = ((int)blockIdx.x + grp * (int)gridDim.x) * kTileRows + er;  // row of the next tile's scale
  // (kept in fp16 until first used, so the loads stay in flight across the dependency wait)
  __half sc0n = tiles_g > 0 && nn < N ? scales[nn] : __ushort_as_half(0);
  __half sc1n = RT == 2 && tiles_g > 0 && half_n + nn < N ? scales[half_n + nn] : __ushort_as_half(0);

  pdl_wait();  // activations, tokens and sums of squares come from earlier launches

  if (P.xcontig) {  // all M rows in one request (the issue cost is per request)
    if (tid == 0) bulk_load(xsm, rowp_s[0], static_cast<uint32_t>(M) * kend * 2, xbar);
  } else if (tid < M && (rmode_s[tid] == HM_SRC_F16 || rmode_s[tid] == HM_SRC_RMS)) {
    bulk_load(xsm + tid * L.xp, rowp_s[tid] + 2 * k0, kend * 2, xbar);  // one row per thread
  }
  if (any_emb) {
    // ---- embedding rows: token id -> table row and scale (rejected ids -> zero row)
    if (tid < M && rmode_s[tid] == HM_SRC_EMB) {
      const int m = tid;
      int row, sel;
      const hm_row_src& s = src_of(d, m, row, sel);
      const int64_t id = s.tok[(int64_t)row * s.tok_ld + s.tok_col] + s.tok_off;
      if (id < 0 || id >= s.erows) {
        report_error(err, HM_ERR_BADINDEX);
        rmode_s[m] = -1;
      } else {
        rowp_s[m] = reinterpret_cast<const uint8_t*>(s.etab + id * (int64_t)K);
        esc_s[m] = __half2float(reinterpret_cast<const __half*>(s.escale)[id]);
      }
    }
    named_bar(kBarCons, kCons);
    for (int m = 0; m < M; ++m) {
      const int mode = rmode_s[m];
      uint8_t* xr = xsm + m * L.xp;
      if (mode == HM_SRC_EMB) {
        const uint8_t* base = rowp_s[m] + k0;
        for (int c = tid; c < ctail; c += kCons) cp_async8(xr + c * 16, base + 8 * c);
      } else if (mode < 0) {
        for (int c = tid; c < ctail; c += kCons) *reinterpret_cast<uint4*>(xr + c * 16) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  // ---- RMSNorm 1/rms of RMS rows from the producers' ss partials, while the copies fly.
  // Every CTA reads the same few KB of partials, so the read pattern matters: with one
  // source of consecutive rows (the decode layout) each thread loads whole 16-byte
  // groups of rows of its partial tiles (one request per 4 rows instead of one per
  // value), and the CTA reduces them; otherwise one warp per row.
  const hm_row_src& s0 = d.src[0];
  const bool rms_vec = !d.interleave && s0.mode == HM_SRC_RMS && s0.row_mul == 1 && (s0.row_add & 3) == 0 &&
                       (s0.ss_ld & 3) == 0 && (reinterpret_cast<uintptr_t>(s0.ss) & 15u) == 0;
  if (rms_vec) {
    constexpr int NV = (MROWS + 3) / 4;
    const int nv = (M + 3) / 4;
    float a[4 * NV];
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) a[i] = 0.f;
    const float* ss = s0.ss + s0.row_add;
    const int tiles = s0.ss_tiles;
    const int64_t ld = s0.ss_ld;
    // the first group's threads only: the same summation order for every kernel shape
    for (int t = tid; t < (tid < kGT ? tiles : 0); t += kGT) {
      const float4* p4 = reinterpret_cast<const float4*>(ss + (int64_t)t * ld);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (j < nv) {
          const float4 v = p4[j];
          a[4 * j] += v.x;
          a[4 * j + 1] += v.y;
          a[4 * j + 2] += v.z;
          a[4 * j + 3] += v.w;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) a[i] = warp_sum(a[i]);
    float* part = red_s;  // [4 warps][MROWS], free until the first tile
    if (lane == 0 && tid < kGT) {
#pragma unroll
      for (int i = 0; i < 4 * NV; ++i)
        if (i < MROWS) part[warp * MROWS + i] = a[i];
    }
    named_bar(kBarCons, kCons);
    if (tid < M) {
      const float tot = ((part[tid] + part[MROWS + tid]) + part[2 * MROWS + tid]) + part[3 * MROWS + tid];
      inv_s[tid] = 1.0f / sqrtf(tot / static_cast<float>(s0.dim) + s0.eps);
    }
  } else {
    for (int m = warp; m < M; m += kCons / 32) {
      int row, sel;
      const hm_row_src& s = src_of(d, m, row, sel);
      if (s.mode != HM_SRC_RMS) continue;
      const float a = warp_sum_partials(s.ss, s.ss_tiles, s.ss_ld, row, lane);
      if (lane == 0) inv_s[m] = 1.0f / sqrtf(a / static_cast<float>(s.dim) + s.eps);
    }
  }
  cp_async_wait_all();
  mbar_wait_ab(xbar, 0, err, abort_s);
  named_bar(kBarCons, kCons);

  // ---- in-place transforms.  RMSNorm, fp16(fp16(x * inv) * gamma): chunk-outer with the
  // 8 rows of a group loaded together, so each thread has 8 independent load / math /
  // store chains in flight (a row-outer loop is latency-bound at 4 warps per CTA).
  bool any_rms = false;
  for (int m = 0; m < M; ++m) any_rms |= rmode_s[m] == HM_SRC_RMS;
  if (any_rms && !xf_loop) {
    // per-row parameters in registers (the stores below go through a byte pointer,
    // which would otherwise force every shared-memory scalar to be re-read)
    float invr[MROWS];
    uint32_t onmask = 0, selmask = 0;
#pragma unroll
    for (int m = 0; m < MROWS; ++m) {
      const bool on = m < M && rmode_s[m] == HM_SRC_RMS;
      invr[m] = on ? inv_s[m] : 0.f;
      onmask |= on ? (1u << m) : 0u;
      selmask |= (on && rsel_s[m]) ? (1u << m) : 0u;
    }
    uint4* const x4 = reinterpret_cast<uint4*>(xsm);
    const int xp4 = L.xp / 16;
    for (int c = tid; c < cpr && 8 * c < kend; c += kCons) {
      const uint4 gv0 = reinterpret_cast<const uint4*>(gam_s)[c];
      const uint4 gv1 = g1 ? reinterpret_cast<const uint4*>(gam_s + kspan)[c] : gv0;
#pragma unroll
      for (int m0 = 0; m0 < MROWS; m0 += 8) {
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if ((onmask >> (m0 + i)) & 1u) v[i] = x4[(m0 + i) * xp4 + c];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + i;
          if (!((onmask >> m) & 1u)) continue;
          const float inv = invr[m];
          const uint4 gv = ((selmask >> m) & 1u) ? gv1 : gv0;
          uint4 r;
          r.x = rms_h2(v[i].x, gv.x, inv);
          r.y = rms_h2(v[i].y, gv.y, inv);
          r.z = rms_h2(v[i].z, gv.z, inv);
          r.w = rms_h2(v[i].w, gv.w, inv);
          x4[m * xp4 + c] = r;
        }
      }
    }
  }
  if (any_emb) {  // int8 -> fp16 embedding rows
    for (int m = 0; m < M; ++m) {
      if (rmode_s[m] != HM_SRC_EMB) continue;
      uint8_t* xr = xsm + m * L.xp;
      const float sc = esc_s[m];
      for (int c = tid; c < cpr && 8 * c < kend; c += kCons) {
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

  // ---- tiles: warp gw of a group consumes box gw of every stage of the group's ring
  // (row block gw % RT, k slice gw / RT); groups without tiles are done
  if (tiles_g == 0) return;
  const int g = lane >> 2, t = lane & 3;
  const int rot = t >> 1;  // lanes t >= 2 read their activation chunks rotated by two
  const int ksub = gw / RT;
  uint8_t* const gring = ring + grp * nst * kStage;
  uint64_t* const gfull = full + grp * kMaxNST;
  uint64_t* const gempty = empty + grp * kMaxNST;
  float* const red_g = red_s + grp * kGW * kTileRows * MP;
  // epilogue ownership: thread -> (row r of the 16 (er), rows m = em0, em0 + 8, ...)
  // in-loop RMSNorm: 1/rms of this lane's activation rows (8j + g); padding rows are zeros
  float ivr[MT];
#pragma unroll
  for (int j = 0; j < MT; ++j) ivr[j] = (xf_loop && 8 * j + g < M) ? inv_s[8 * j + g] : 0.f;
  const uint4* const gam4 = reinterpret_cast<const uint4*>(gam_s);
  int slot = 0, round = 0;  // ring position of the next stage
  for (int ti = 0; ti < tiles_g; ++ti) {
    const int tile = (int)blockIdx.x + (grp + ti * G) * (int)gridDim.x;
    const int n0 = tile * kTileRows + er;
    const float sc0 = __half2float(sc0n), sc1 = __half2float(sc1n);
    if (ti + 1 < tiles_g) {
      nn += G * (int)gridDim.x * kTileRows;
      sc0n = nn < N ? scales[nn] : __ushort_as_half(0);
      if (RT == 2) sc1n = half_n + nn < N ? scales[half_n + nn] : __ushort_as_half(0);
    }
    float acc[MT][4];
#pragma unroll
    for (int j = 0; j < MT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int st = 0; st < per_tile; ++st) {
      mbar_wait_ab(&gfull[slot], round & 1, err, abort_s);  // on timeout: carry on, error flagged
      const uint8_t* wb = gring + slot * kStage + gw * kBoxBytes;
      const uint4 lo0 = *reinterpret_cast<const uint4*>(wb + g * kBox + (((2 * t + rot) ^ g) << 4));
      const uint4 lo1 = *reinterpret_cast<const uint4*>(wb + g * kBox + (((2 * t + 1 - rot) ^ g) << 4));
      const uint4 hi0 = *reinterpret_cast<const uint4*>(wb + (g + 8) * kBox + (((2 * t + rot) ^ g) << 4));
      const uint4 hi1 = *reinterpret_cast<const uint4*>(wb + (g + 8) * kBox + (((2 * t + 1 - rot) ^ g) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&gempty[slot]);  // this warp's box is in registers now
      if (++slot == nst) {
        slot = 0;
        ++round;
      }
      const uint32_t wa[8] = {lo0.x, lo0.y, lo0.z, lo0.w, lo1.x, lo1.y, lo1.z, lo1.w};
      const uint32_t wc[8] = {hi0.x, hi0.y, hi0.z, hi0.w, hi1.x, hi1.y, hi1.z, hi1.w};
      const int cb = (st * KS + ksub * kBox) / 8;  // first activation chunk of this box
      uint32_t xw[MT][16];
#pragma unroll
      for (int j = 0; j < MT; ++j) {
        const uint8_t* xr = xsm + (8 * j + g) * L.xp;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 v = *reinterpret_cast<const uint4*>(xr + (cb + 4 * t + ((i + 2 * rot) & 3)) * 16);
          xw[j][4 * i + 0] = v.x;
          xw[j][4 * i + 1] = v.y;
          xw[j][4 * i + 2] = v.z;
          xw[j][4 * i + 3] = v.w;
        }
      }
      if (xf_loop) {  // fp16(fp16(x * inv) * gamma), the same rounding as the shared-memory pass
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 gv = gam4[cb + 4 * t + ((i + 2 * rot) & 3)];
#pragma unroll
          for (int j = 0; j < MT; ++j) {
            xw[j][4 * i + 0] = rms_h2(xw[j][4 * i + 0], gv.x, ivr[j]);
            xw[j][4 * i + 1] = rms_h2(xw[j][4 * i + 1], gv.y, ivr[j]);
            xw[j][4 * i + 2] = rms_h2(xw[j][4 * i + 2], gv.z, ivr[j]);
            xw[j][4 * i + 3] = rms_h2(xw[j][4 * i + 3], gv.w, ivr[j]);
          }
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
    // ---- partial sums of the group's four warps -> red_g[warp][row][m]
    float* rw = red_g + gw * kTileRows * MP;
#pragma unroll
    for (int j = 0; j < MT; ++j) {
      const int m = 8 * j + 2 * t;
      rw[g * MP + m] = acc[j][0];
      rw[g * MP + m + 1] = acc[j][1];
      rw[(g + 8) * MP + m] = acc[j][2];
      rw[(g + 8) * MP + m + 1] = acc[j][3];
    }
    group_bar<GR>(grp);
    // value of (row block b, row r, activation row m): warps b, b+RT, ... summed in order
    auto tile_sum = [&](int b, int r, int m) {
      float a = 0.f;
#pragma unroll
      for (int w = b; w < kGW; w += RT) a += red_g[(w * kTileRows + r) * MP + m];
      return a;
    };

    // ---- split-K (only when the activations did not fit): last CTA sums partials in split order
    bool owner = true;
    if (P.nsplit > 1 && P.cluster) {
      // ---- cluster split: every k-range keeps its partial tile in its own shared memory;
      // rank 0 (k-range 0) sums them through DSMEM in split order -- the arithmetic of the
      // workspace path below -- and runs the epilogue; the others wait until it has read
      // their partial (their shared memory must outlive the reads)
      const int per = RT * kTileRows * M;
      for (int i = gtid; i < per; i += kGT) {
        const int b = i / (kTileRows * M), r = (i / M) % kTileRows, m = i % M;
        cpart_s[i] = tile_sum(b, r, m);
      }
      group_bar<GR>(grp);
      if (cluster_ctarank() != 0) {
        if (gtid == 0) {
          fence_acq_rel_cluster();
          mbar_arrive_dsmem(dsmem_addr(cready, 0));
          mbar_wait_cluster(cdone, ti & 1, err);
        }
        group_bar<GR>(grp);
        owner = false;
      } else {
        if (gtid == 0) mbar_wait_cluster(cready, ti & 1, err);
        group_bar<GR>(grp);
        for (int i = gtid; i < per; i += kGT) {
          const int b = i / (kTileRows * M), r = (i / M) % kTileRows, m = i % M;
          float v[kMaxCSplit];
#pragma unroll
          for (int sp = 0; sp < kMaxCSplit; ++sp)
            v[sp] = sp >= P.nsplit ? 0.f : (sp == 0 ? cpart_s[i] : ld_dsmem_f32(dsmem_addr(cpart_s + i, sp)));
          float a = 0.f;
#pragma unroll
          for (int sp = 0; sp < kMaxCSplit; ++sp)
            if (sp < P.nsplit) a += v[sp];
          red_g[(b * kTileRows + r) * MP + m] = a;  // warp-b slot now holds the full sum
        }
        group_bar<GR>(grp);  // every DSMEM read of this tile has returned
        if (gtid == 0)
          for (int sp = 1; sp < P.nsplit; ++sp) mbar_arrive_dsmem(dsmem_addr(cdone, sp));
      }
    } else if (P.nsplit > 1) {
      float* ws = wsp;
      const int per = RT * kTileRows * M;
      float* mine = ws + ((int64_t)split * P.ntiles + tile) * per;
      for (int i = gtid; i < per; i += kGT) {
        const int b = i / (kTileRows * M), r = (i / M) % kTileRows, m = i % M;
        mine[i] = tile_sum(b, r, m);
      }
      __threadfence();
      group_bar<GR>(grp);
      if (gtid == 0) flag_s[grp] = (atomicAdd(&counters[tile], 1) == P.nsplit - 1);
      group_bar<GR>(grp);
      owner = flag_s[grp] != 0;
      if (owner) {
        __threadfence();
        for (int i = gtid; i < per; i += kGT) {
          const int b = i / (kTileRows * M), r = (i / M) % kTileRows, m = i % M;
          float a = 0.f;
          for (int sp = 0; sp < P.nsplit; ++sp) a += __ldcg(ws + ((int64_t)sp * P.ntiles + tile) * per + i);
          red_g[(b * kTileRows + r) * MP + m] = a;  // warp-b slot now holds the full sum
        }
        if (gtid == 0) counters[tile] = 0;
        group_bar<GR>(grp);
      }
    }
    auto value = [&](int b, int r, int m) {
      return P.nsplit > 1 ? red_g[(b * kTileRows + r) * MP + m] : tile_sum(b, r, m);
    };

    // ---- epilogues (the owner of the tile only)
    if (owner) {
      if (epi == HM_EPI_STORE) {
        __half* y = yout;
        const __half* res = resid;
        const int n = n0;
#pragma unroll
        for (int q = 0; q < MT; ++q) {
          const int m = em0 + 8 * q;
          float sq = 0.f;
          if (m < M && n < N) {
            __half v = __float2half_rn(value(0, er, m) * sc0);
            if (res) v = hadd_rn(v, res[(int64_t)m * ldres + n]);
            y[(int64_t)m * ldy + n] = v;
            const float vf = __half2float(v);
            sq = vf * vf;
          }
          if (ss_out) {  // 16 consecutive lanes share m: sum over the tile's 16 columns
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            if (er == 0 && m < M) ss_out[(int64_t)tile * ss_ld + m] = sq;
          }
        }
      } else if (epi == HM_EPI_ROPE_KV) {
        const int hd = rp.hd, qw = rp.qw, kw = rp.kw;
        __half* qo = rp.qo;
        __half* kc = rp.kc;
        __half* vc = rp.vc;
        // the pair (2i, 2i+1) is handled by the thread of row 2i; its partner row's
        // scale comes from the neighbouring lane
        const float sc_next = __shfl_down_sync(0xffffffffu, sc0, 1);
#pragma unroll
        for (int q = 0; q < MT; ++q) {
          const int m = em0 + 8 * q;
          const int n = n0;
          if ((er & 1) || m >= M || n >= N) continue;
          const float x0 = __half2float(__float2half_rn(value(0, er, m) * sc0));
          const float x1 = __half2float(__float2half_rn(value(0, er + 1, m) * sc_next));
          const int64_t p = rp.pos[m];
          const int bb = m / rp.S;
          if (p < 0 || p >= rp.L || p >= rp.rope_rows) {
            report_error(err, HM_ERR_BADINDEX);
            continue;
          }
          const int dh = n % hd;
          if (n < qw + kw) {
            const float* cs = rp.rope + (p * (hd / 2) + dh / 2) * 2;
            const float c = cs[0], sn = cs[1];
            const __half y0 = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
            const __half y1 = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
            __half* dst;
            if (n < qw) {
              dst = qo + (int64_t)m * qw + n;
            } else {
              const int kh = (n - qw) / hd;
              dst = kc + (((int64_t)bb * rp.Hk + kh) * rp.L + p) * hd + dh;
            }
            dst[0] = y0;
            dst[1] = y1;
          } else {
            const int kh = (n - qw - kw) / hd;
            __half* dst = vc + (((int64_t)bb * rp.Hk + kh) * rp.L + p) * hd + dh;
            dst[0] = __float2half_rn(x0);
            dst[1] = __float2half_rn(x1);
          }
        }
      } else {  // HM_EPI_SILU: row block 0 = w1 (a), row block 1 = w3 (b)
        __half* y = yout;
#pragma unroll
        for (int q = 0; q < MT; ++q) {
          const int m = em0 + 8 * q;
          if (m >= M) continue;
          const __half a = __float2half_rn(value(0, er, m) * sc0);
          const __half bv = __float2half_rn(value(1, er, m) * sc1);
          const float af = __half2float(a);
          const __half sl = __float2half_rn(__fdiv_rn(af, __fadd_rn(1.0f, expf(-af))));
          y[(int64_t)m * ldy + n0] = hmul_rn(sl, bv);
        }
      }
    }
    group_bar<GR>(grp);  // red_g is reused by the next tile
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
  int n, k, kind;
  bool operator==(const MapKey& o) const { return p == o.p && n == o.n && k == o.k && kind == o.kind; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (static_cast<size_t>(k.n) * 1000003u) ^ (static_cast<size_t>(k.k) << 20) ^
           (static_cast<size_t>(k.kind) << 40);
  }
};

// Tensor map of the int8 weights [N, K] (row pitch K bytes), 128B swizzle.
//  kind 0: 2-D {K, N}, box 128 x 16 (2 KB): four requests per 8 KB stage.
//  kind 1: 3-D {128, N, K/128} (k within a 128-byte chunk, row, chunk; the chunk stride is
//          128 bytes), box {128, 16, 4}: one request per stage, laid out in shared memory as
//          [chunk][row][128 bytes] -- the four 2-D boxes of kind 0, in the same order.
//  kind 2: 4-D {128, N/2, 2, K/128} for the fused w1|w3 matrix (row within a half, half,
//          chunk), box {128, 16, 2, 2}: [chunk][half][row][128 bytes], again kind 0's layout
//          for the SiLU epilogue (w1 rows, w3 rows of the same k chunk side by side).
// Kinds 1 and 2 need K % 128 == 0 (a chunk must not run into the next row: out-of-range
// k would otherwise read the next row's bytes instead of the zero fill).
bool weight_map(const int8_t* w, int N, int K, int kind, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{w, N, K, kind};
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
  if (kind != 0 && (K % kBox || (kind == 2 && N % (2 * kTileRows)))) return false;
  CUtensorMap m;
  const cuuint64_t k = static_cast<cuuint64_t>(K), n = static_cast<cuuint64_t>(N);
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r;
  if (kind == 0) {
    cuuint64_t dims[2] = {k, n};
    cuuint64_t strides[1] = {k};
    cuuint32_t box[2] = {kBox, kTileRows};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (kind == 1) {
    cuuint64_t dims[3] = {kBox, n, k / kBox};
    cuuint64_t strides[2] = {k, kBox};
    cuuint32_t box[3] = {kBox, kTileRows, 4};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[4] = {kBox, n / 2, 2, k / kBox};
    cuuint64_t strides[3] = {k, (n / 2) * k, kBox};
    cuuint32_t box[4] = {kBox, kTileRows, 2, 2};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
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

int dev_attr(cudaDeviceAttr a, int dflt) {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  return cudaDeviceGetAttribute(&v, a, dev) == cudaSuccess && v > 0 ? v : dflt;
}
int smem_per_sm() {
  static const int v = dev_attr(cudaDevAttrMaxSharedMemoryPerMultiprocessor, 228 * 1024);
  return v;
}
int smem_reserved_per_cta() {
  static const int v = dev_attr(cudaDevAttrReservedSharedMemoryPerBlock, 1024);
  return v;
}

int ntiles_of(int N, int epi) {
  return epi == HM_EPI_SILU ? (N / 2) / kTileRows : (N + kTileRows - 1) / kTileRows;
}

double env_or(const char* name, double dflt) {
  const char* e = getenv(name);
  return e ? atof(e) : dflt;
}

int mrows_of(int M) { return M <= 8 ? 8 : (M <= 16 ? 16 : 32); }

// K rounded up to whole stages (the tail is zero-filled by TMA and masked for x)
int padded_k(int K, int epi) { return (K + ks_of(epi) - 1) / ks_of(epi) * ks_of(epi); }

// The widest k-range (fewest splits) whose staged activations fit the budget.
int auto_kspan(int M, int K, int epi) {
  const int ks = ks_of(epi), kp = padded_k(K, epi), mr = mrows_of(M);
  static const int budget = static_cast<int>(env_or("HM_GEMV_X_BUDGET", 136 * 1024));
  for (int s = 1; s <= kp / ks; ++s) {
    if ((kp / ks) % s) continue;
    const int span = kp / s;
    if (mr * (span * 2 + 16) <= budget) return span;
  }
  return ks;
}

// One wave of CTAs, tiles strided over the grid.  CTAs per SM: enough for one tile per CTA
// when the shape has more tiles than SMs and the activations are short enough for up to
// four CTAs with a ring of at least four stages; otherwise up to two CTAs (what the shared
// memory allows) with the default ring, deepened into the memory they leave free: the
// bytes in flight per SM bound its weight stream (bandwidth = bytes in flight / memory
// latency), which matters when a long activation row leaves room for one CTA per SM only.
template <int MT, int EPI>
void choose_occupancy(const GemvParams& p, int* per_sm_out, int* nst_out) {
  static const int cap = static_cast<int>(env_or("HM_GEMV_CTAS_PER_SM", 4));
  static const int deep = static_cast<int>(env_or("HM_GEMV_DEEP_RING", 1));
  const int units = p.ntiles * p.nsplit;
  const int want = std::max(2, (units + sm_count() - 1) / sm_count());
  auto lay = [&](int n) { return smem_layout(p.kspan, 8 * MT, p.has_gamma, p.xcontig, n).total; };
  for (int ps = std::min(cap, want); ps >= 1; --ps) {
    const int limit = std::min(smem_per_sm() / ps - smem_reserved_per_cta(), 227 * 1024);
    int n = kNST;
    if (ps > 2) {
      n = kMaxNST;
      while (n >= 4 && lay(n) > limit) --n;
      if (n < 4) continue;
    } else {
      if (lay(n) > limit) continue;
      if (deep)
        while (n < kMaxNST && lay(n + 1) <= limit) ++n;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_i8_kernel<MT, EPI, 1>, threads_of(1), lay(n)) !=
            cudaSuccess ||
        occ < ps)
      continue;
    *per_sm_out = ps;
    *nst_out = n;
    return;
  }
  *per_sm_out = 1;
  *nst_out = kNST;
}

// Split of K over the CTAs of a cluster (1 = none) for a shape whose activations fit one
// CTA: the split that minimises the stages streamed by the busiest CTA, plus a reduction
// cost per split tile.  It pays when there are too few tiles for the CTAs the GPU holds
// (a long K and a short N) or when a few CTAs would stream a second whole tile.
template <int MT, int EPI>
int choose_cluster_split(const GemvParams& p) {
  constexpr int kRedStages = 4;  // a DSMEM reduction round costs about as much as four stages
  const int stages = p.kspan / ks_of(EPI >= 0 ? EPI : p.d.epi);  // the whole K in one k-range (nsplit 1)
  int best = 1;
  long best_cost = -1;
  for (int sp = 1; sp <= kMaxCSplit; sp *= 2) {
    if (stages % sp) continue;
    GemvParams q = p;
    q.kspan = p.kspan / sp;
    q.nsplit = sp;
    q.xcontig = sp == 1 ? p.xcontig : 0;
    if (smem_layout(q.kspan, 8 * MT, q.has_gamma, q.xcontig).total > 227 * 1024) continue;
    int per_sm = 1, nst = kNST;
    choose_occupancy<MT, EPI>(q, &per_sm, &nst);
    const int J = std::max(1, std::min(q.ntiles, per_sm * sm_count() / sp));
    const long tiles_per_cta = (q.ntiles + J - 1) / J;
    const long cost = tiles_per_cta * (stages / sp + (sp > 1 ? kRedStages : 0));
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

template <int MT, int EPI, int GR>
cudaError_t configure_kernel() {
  static int configured = 0;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemv_i8_kernel<MT, EPI, GR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return e;
    hm_carveout(gemv_i8_kernel<MT, EPI, GR>);
    configured = 1;
  }
  return cudaSuccess;
}

template <int MT, int EPI, int GR>
cudaError_t launch_grid(const CUtensorMap& map, const GemvParams& p, int J, int smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(J, p.nsplit);
  cfg.blockDim = dim3(threads_of(GR));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (p.d.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = p.nsplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemv_i8_kernel<MT, EPI, GR>, map, p);
}

// Consumer groups of the wide kernel: four at 8 rows; three at 16 rows, whose MMA loop
// needs more registers than a 17-warp CTA leaves per thread.
template <int MT>
constexpr int wide_groups() { return MT == 1 ? kMaxGroups : 3; }

// The wide kernel (8 or 16 rows, one k-range): one CTA per SM, as many consumer groups
// as the SM has tiles (up to wide_groups), each with the deepest ring that fits.
// Returns false when the shape does not fit it (the narrow kernel runs instead).
template <int MT, int EPI>
bool wide_shape(GemvParams& p, int* J, int* smem) {
  constexpr int GRW = wide_groups<MT>();
  if (configure_kernel<MT, EPI, GRW>() != cudaSuccess) return false;  // before the occupancy query
  const int nsm = sm_count();
  *J = std::min(p.ntiles, nsm);
  for (int G = std::min(GRW, (p.ntiles + *J - 1) / *J); G >= 1; --G) {
    int n = kMaxNST;
    while (n >= 2 && smem_layout(p.kspan, 8 * MT, p.has_gamma, p.xcontig, n, G).total > 227 * 1024) --n;
    if (n < 2) continue;
    int occ = 0;
    const int sm = smem_layout(p.kspan, 8 * MT, p.has_gamma, p.xcontig, n, G).total;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_i8_kernel<MT, EPI, GRW>,
                                                      threads_of(GRW), sm) != cudaSuccess ||
        occ < 1)
      return false;
    p.groups = G;
    p.nst = n;
    *smem = sm;
    return true;
  }
  return false;
}

template <int MT, int EPI>
cudaError_t launch_one(const CUtensorMap& map, const GemvParams& p0, cudaStream_t st) {
  GemvParams p = p0;
  p.groups = 1;
  cudaError_t e = configure_kernel<MT, EPI, 1>();
  if (e != cudaSuccess) return e;
  if (p.cluster < 0) {  // automatic cluster split (whole-K k-range requested)
    const int sp = choose_cluster_split<MT, EPI>(p);
    p.cluster = sp > 1;
    if (sp > 1) {
      p.kspan /= sp;
      p.nsplit = sp;
      p.xcontig = 0;
    }
  }
  int per_sm = 1;
  choose_occupancy<MT, EPI>(p, &per_sm, &p.nst);
  // HM_GEMV_WIDE: 1 (default) the wide kernel when the narrow one cannot give every tile
  // its own CTA (some CTAs would stream a second tile after their first), 2 for every
  // 8- or 16-row launch with one k-range, 0 never.  (A wide CTA cannot share its SM with
  // the previous launch's tail, so short launches that fit the narrow kernel keep it.)
  static const int wide = static_cast<int>(env_or("HM_GEMV_WIDE", 1));
  if constexpr (MT <= 2) {
    if (p.nsplit == 1 && !p.cluster && (wide == 2 || (wide == 1 && p.ntiles > per_sm * sm_count()))) {
      GemvParams q = p;
      int J = 0, smem = 0;
      if (wide_shape<MT, EPI>(q, &J, &smem))
        return launch_grid<MT, EPI, wide_groups<MT>()>(map, q, J, smem, st);
    }
  }
  const int smem = smem_layout(p.kspan, 8 * MT, p.has_gamma, p.xcontig, p.nst).total;
  int J = per_sm * sm_count() / p.nsplit;
  if (J < 1) J = 1;
  if (J > p.ntiles) J = p.ntiles;
  return launch_grid<MT, EPI, 1>(map, p, J, smem, st);
}

template <int EPI>
cudaError_t launch_mt(int mt, const CUtensorMap& map, const GemvParams& p, cudaStream_t st) {
  if (mt == 1) return launch_one<1, EPI>(map, p, st);
  if (mt == 2) return launch_one<2, EPI>(map, p, st);
  return launch_one<4, EPI>(map, p, st);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int gemv_box_on() {
  static const int on = static_cast<int>(env_or("HM_GEMV_BOX", 1));
  return on;
}

}  // namespace

extern "C" int hm_gemv_box_form(const int8_t* w, int N, int K, int epi) {
  if (!w || N < 1 || K < 16 || K % 16 || (epi == HM_EPI_SILU && N % (2 * kTileRows))) return HM_EARG;
  CUtensorMap m;
  if (gemv_box_on() && weight_map(w, N, K, epi == HM_EPI_SILU ? 2 : 1, &m)) return 1;
  return weight_map(w, N, K, 0, &m) ? 0 : HM_EARG;
}


extern "C" int hm_gemv_pick_kspan(int M, int N, int K, int epi, int kspan) {
  (void)N;
  if (kspan > 0) return kspan;
  return auto_kspan(M, K, epi);
}

extern "C" int hm_gemv_counters(int N, int epi) { return ntiles_of(N, epi); }

extern "C" size_t hm_gemv_workspace_bytes(int M, int N, int K, int epi, int kspan) {
  const int ks = hm_gemv_pick_kspan(M, N, K, epi, kspan);
  if (ks <= 0) return 0;
  const int nsplit = padded_k(K, epi) / ks;
  if (nsplit <= 1) return 0;
  return static_cast<size_t>(nsplit) * ntiles_of(N, epi) * rt_of(epi) * kTileRows * M * sizeof(float);
}

extern "C" int hm_gemv_i8_fused(const hm_gemv_desc* d, hm_stream_t stream) {
  if (!d || !d->w || !d->s || d->M < 1 || d->M > kMaxM || d->N < 1 || d->K < 16 || d->K % 16) return HM_EARG;
  if (!aligned16(d->w)) return HM_EARG;
  if (d->epi == HM_EPI_SILU && (d->N % (2 * kTileRows) || !d->y)) return HM_EARG;
  if (d->epi == HM_EPI_STORE && !d->y) return HM_EARG;
  if (d->epi == HM_EPI_STORE && d->ss_out && d->N % kTileRows) return HM_EARG;
  if (d->epi == HM_EPI_ROPE_KV &&
      (!d->rope || !d->pos || !d->q_out || !d->kc || !d->vc || d->hd % kTileRows || d->S < 1 ||
       d->N != (d->Hq + 2 * d->Hk) * d->hd))
    return HM_EARG;
  int has_gamma = 0;
  for (int i = 0; i < (d->interleave ? 2 : 1); ++i) {
    const hm_row_src& s = d->src[i];
    if (s.mode == HM_SRC_EMB) {
      if (!s.etab || !s.escale || !s.tok || (reinterpret_cast<uintptr_t>(s.etab) & 7u)) return HM_EARG;
    } else {
      if (!s.x || !aligned16(s.x) || (s.ldx % 8)) return HM_EARG;
      if (s.mode == HM_SRC_RMS) {
        if (!s.ss || !s.gamma || !aligned16(s.gamma) || s.dim <= 0) return HM_EARG;
        has_gamma = d->interleave ? 2 : 1;
      }
    }
  }
  GemvParams p;
  p.d = *d;
  p.has_gamma = has_gamma;
  const int kpad = padded_k(d->K, d->epi);
  // kspan < 0: K split over -kspan CTAs of a cluster (2, 4 or 8), reduced in DSMEM
  const int csplit = d->kspan < 0 ? -d->kspan : 0;
  if (csplit && (csplit > kMaxCSplit || (csplit & (csplit - 1)) || (kpad / ks_of(d->epi)) % csplit)) return HM_EARG;
  p.kspan = csplit ? kpad / csplit : hm_gemv_pick_kspan(d->M, d->N, d->K, d->epi, d->kspan);
  if (p.kspan <= 0 || p.kspan % ks_of(d->epi) || kpad % p.kspan) return HM_EARG;
  if (smem_layout(p.kspan, mrows_of(d->M), has_gamma).total > 227 * 1024) return HM_EARG;
  p.nsplit = kpad / p.kspan;
  // automatic k-range with the whole K in one CTA: with HM_GEMV_CSPLIT=1 the launch may
  // still split it over a cluster when a stage-count model says that balances the CTAs
  // better.  Off by default: measured slower on the decode shapes (a cluster starts only
  // when all of its CTAs fit at once, which delays it behind the previous launch's tail,
  // and a DSMEM reduction round costs more than the stages it saves).
  static const int csplit_auto = static_cast<int>(env_or("HM_GEMV_CSPLIT", 0));
  p.cluster = csplit > 1 ? 1 : (d->kspan == 0 && p.nsplit == 1 && csplit_auto ? -1 : 0);
  {
    // one bulk copy for all rows (HM_GEMV_XCONTIG=1): one fp16/RMS source, consecutive
    // rows, row pitch K, whole K in one k-range, 16-byte aligned block start.  Off by
    // default: the unpadded row pitch (a multiple of 128 bytes) puts two rows of every
    // quarter-warp's fragment loads on the same banks, and the per-row copies, issued
    // by one thread each, measured faster.
    static const int contig_on = static_cast<int>(env_or("HM_GEMV_XCONTIG", 0));
    const hm_row_src& s0 = d->src[0];
    const char* blk = reinterpret_cast<const char*>(s0.x) + static_cast<int64_t>(s0.row_add) * s0.ldx * 2;
    p.xcontig = contig_on && !d->interleave && (s0.mode == HM_SRC_F16 || s0.mode == HM_SRC_RMS) &&
                s0.row_mul == 1 && s0.ldx == d->K && p.nsplit == 1 && p.kspan == d->K &&
                (reinterpret_cast<uintptr_t>(blk) & 15u) == 0;
    static const int xf_on = static_cast<int>(env_or("HM_GEMV_XFLOOP", 1));
    p.xf_loop = xf_on && !d->interleave && s0.mode == HM_SRC_RMS;
  }
  p.ntiles = ntiles_of(d->N, d->epi);
  if (p.nsplit > 1 && p.cluster != 1) {
    if (!d->ws || !d->counters || d->n_counters < p.ntiles ||
        d->ws_bytes < hm_gemv_workspace_bytes(d->M, d->N, d->K, d->epi, p.kspan))
      return HM_EARG;
  }
  // one weight request per stage (HM_GEMV_BOX=1, the default) where the map allows it,
  // else four 2-D boxes; both fill the ring identically, so the results are the same
  CUtensorMap map;
  p.box = 0;
  if (gemv_box_on() && weight_map(d->w, d->N, d->K, d->epi == HM_EPI_SILU ? 2 : 1, &map)) {
    p.box = 1;
  } else if (!weight_map(d->w, d->N, d->K, 0, &map)) {
    return HM_EARG;
  }
  const int mt = d->M <= 8 ? 1 : (d->M <= 16 ? 2 : 4);
  cudaError_t e;
  static const int generic = static_cast<int>(env_or("HM_GEMV_ONE_KERNEL", 1));
  if (generic && (d->epi == HM_EPI_STORE || d->epi == HM_EPI_ROPE_KV || d->epi == HM_EPI_SILU)) {
    e = launch_mt<-1>(mt, map, p, stream);
    return e == cudaSuccess ? HM_OK : static_cast<int>(e);
  }
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
    case 5: return offsetof(hm_gemv_desc, l2_keep);
    case 6: return sizeof(hm_conv_desc);
    case 7: return offsetof(hm_conv_desc, B);
    case 8: return offsetof(hm_conv_desc, scale);
    case 9: return offsetof(hm_conv_desc, bn);
    default: return 0;
  }
}

extern "C" const char* hm_version(void) { return "heartmula_b200 0.4 sm_100a"; }
