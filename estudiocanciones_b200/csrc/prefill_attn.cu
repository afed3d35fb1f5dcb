// Causal GQA prefill attention over the static KV cache on the 5th-generation
// tensor cores (sm_100a).
//
// Replaces the prompt branch of the reference's attention in Block.__call__
// (app/engine.py:123-153): for a prompt of P positions the reference expands K/V
// over the query heads (repeat_interleave) and calls SDPA with is_causal.  Here
// K/V are read straight from the cache the RoPE/KV-write step filled, by every
// query head of the KV head's group (through L2; no expanded copy).
//
//   o[b*P + p, h*hd + d] = sum_{j <= p} softmax_j(q_p . k_j * scale) v_j[d]
//
// Work item = 128 query positions of one query head and batch row; K/V tiles of 128
// positions.  Persistent CTAs, one per SM (192 KB of shared memory), each walking the
// items in longest-first order with a stride of the grid; the K/V tile stream, the S
// buffers and the P tile run on across items, so the next item's Q load and first S
// MMAs overlap the current item's last tiles and epilogue.  Warp roles (320 threads):
//   warp 0     TMA producer: each item's Q tile (once the previous item's last S MMA has
//              read the buffer), then its K and V tiles through two separate 2-stage
//              rings (a K slot frees when its S MMA completes, a V slot when its PV MMA
//              does), 128B-swizzled 128 x 64 boxes.
//   warp 1     allocates 512 TMEM columns; one thread issues
//                S_g  = Q K_g^T  (M=128, N=128, K=128; columns 128*(g%2), two buffers)
//                O   += P_g V_g  (M=128, N=128, K=128; columns 256..383; P_g read from
//                                 TMEM columns 384..447, V_g as an MN-major operand)
//              over the global tile sequence g: S_0, S_1, then per tile: O += P_g V_g,
//              S_{g+2} (whatever item it belongs to), so the tensor core computes
//              S_{g+1} and PV_g while the softmax works on S_g.  Descriptors are made
//              once; each operand is one of them plus a constant.
//   warps 2-9  softmax, two threads per query row (TMEM lane = row; warps w and w+4
//              share a lane quarter and take key columns 0-63 / 64-127): scaled,
//              causally masked row max (the two halves swap partial maxima through
//              shared memory) -> p = 2^(s*scale*log2(e) - m) in fp32 (partial row sums
//              l) -> rounded to fp16 pairs and stored to TMEM (tcgen05.st).  The running
//              max m is only raised (and O, l rescaled in TMEM by 2^(m_old - m_new))
//              when the tile's max exceeds it by more than 8 (a factor 2^8): with a
//              stale m, p <= 2^8 and O / l is the same quantity.  Per item the epilogue:
//              O / l -> fp16, staged through this warp's own 32 rows x 64 columns of a
//              shared-memory tile, then written as whole 128-byte row segments.
// Probabilities are rounded to fp16 for the PV product and the row sum is taken over
// the fp32 values (the FA2 rounding scheme).  Masked keys (causal, and cache slots at
// or past P in the diagonal tile, whose V rows are zeroed in shared memory) contribute
// exact zeros, whatever the cache holds there.  Every wait is bounded (HM_ERR_TIMEOUT in
// the caller's error word); before exit the producer waits for its copies and the MMA
// thread for its MMAs.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "hm_common.cuh"
#include "tcgen05.cuh"

namespace {

constexpr int kT = 128;            // query positions per CTA = cache positions per K/V tile
constexpr int kBox = kT * 128;     // one 128-row x 64-column fp16 box, 16 KB
constexpr int kSoftW = 8;         // softmax / epilogue warps
constexpr int kThreads = 64 + 32 * kSoftW;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;    // O accumulator columns 256..383
constexpr uint32_t kPCol = 384;    // P: fp16 pairs of the 128 keys in columns 384..447
constexpr float kRescale = 8.f;    // log2 of the growth the stale max may absorb

// NB: 64-column boxes per head-dim row (hd = 64 NB)
template <int NB>
struct FaSmem {
  uint8_t q[NB][kBox];     // [hd box][128 rows x 64]
  uint8_t k[2][NB][kBox];  // [stage][hd box]
  uint8_t v[2][NB][kBox];  // [stage][hd box]
  uint8_t p[2][kBox];      // the epilogue's staging of O / l (hd 128: per head-dim half)
  float xch[2][2][kT];    // [tile parity][column half][row]: partial row maxima
  float xl[2][kT];        // [column half][row]: partial row sums at an item's end
  uint64_t q_full, q_empty, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full, pv_done, drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct FaParams {
  __half* o;
  int64_t ldo;       // output row stride (elements)
  int B, P, Hq, Hk, L;
  int items;         // ceil(P / 128) * Hq * B
  int causal;        // 1: keys j <= query p (the prompt pass); 0: all keys j < P (the codec's estimator)
  // K/V row of (item b, KV head kh, position t): b * kv_b_rows + kh * kv_h_rows + t, its head-dim
  // columns from kh * kv_h_cols (the cache [B, Hk, L, hd]: Hk*L, L, 0; a fused q|k|v [B*P, ...]:
  // P, 0, hd)
  int kv_b_rows, kv_h_rows, kv_h_cols;
  float scale_log2;  // scale * log2(e)
  int* err;
};

// Work item i in longest-first order: query tile qt (its K/V tiles 0 .. qt when causal, else
// all of them), head h, batch row b; heads of one KV group adjacent, so their K/V tiles meet in L2.
struct Item {
  int qt, h, b, kh, n;
};
HM_DEV Item item_of(const FaParams& p, int i) {
  const int nqt = (p.P + kT - 1) / kT, per = p.Hq * p.B;
  Item it;
  it.qt = nqt - 1 - i / per;
  const int rest = i % per;
  it.h = rest % p.Hq;
  it.b = rest / p.Hq;
  it.kh = it.h / (p.Hq / p.Hk);
  it.n = p.causal ? it.qt + 1 : nqt;
  return it;
}

HM_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                     const __grid_constant__ CUtensorMap kmap,
                                                                     const __grid_constant__ CUtensorMap vmap,
                                                                     const __grid_constant__ FaParams Pp) {
  constexpr int NB = HD / 64;  // head-dim boxes
  constexpr int CW = HD / 2;   // O columns of one softmax warp (the two warps of a lane quarter split hd)
  extern __shared__ uint8_t smem_raw[];
  FaSmem<NB>& sm = *reinterpret_cast<FaSmem<NB>*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = Pp.P;
  const int i0 = static_cast<int>(blockIdx.x), istep = static_cast<int>(gridDim.x), items = Pp.items;
  int* const err = Pp.err;
  volatile int* abort_s = &sm.abort_flag;

  if (tid == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.k_full[i], 1);
      mbar_init(&sm.k_empty[i], 1);
      mbar_init(&sm.v_full[i], 1);
      mbar_init(&sm.v_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
    }
    mbar_init(&sm.p_full, kSoftW);  // one arrival per softmax warp
    mbar_init(&sm.pv_done, 1);
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      int g = 0, k = 0;  // global tile, local item count
      for (int i = i0; i < items; i += istep, ++k) {
        const Item it = item_of(Pp, i);
        if (k > 0) mbar_wait_ab(&sm.q_empty, (k - 1) & 1, err, abort_s);  // previous item's S MMAs done
        mbar_arrive_expect_tx(&sm.q_full, NB * kBox);
        const int qrow = it.b * P + it.qt * kT;
#pragma unroll
        for (int bx = 0; bx < NB; ++bx) tma_load_2d_plain(sm.q[bx], &qmap, it.h * HD + 64 * bx, qrow, &sm.q_full);
        const int krow = it.b * Pp.kv_b_rows + it.kh * Pp.kv_h_rows, kcol = it.kh * Pp.kv_h_cols;
        for (int t = 0; t < it.n; ++t, ++g) {
          const int s = g & 1;
          if (g >= 2) mbar_wait_ab(&sm.k_empty[s], ((g >> 1) - 1) & 1, err, abort_s);
          mbar_arrive_expect_tx(&sm.k_full[s], NB * kBox);
#pragma unroll
          for (int bx = 0; bx < NB; ++bx)
            tma_load_2d_plain(sm.k[s][bx], &kmap, kcol + 64 * bx, krow + t * kT, &sm.k_full[s]);
          if (g >= 2) mbar_wait_ab(&sm.v_empty[s], ((g >> 1) - 1) & 1, err, abort_s);
          mbar_arrive_expect_tx(&sm.v_full[s], NB * kBox);
#pragma unroll
          for (int bx = 0; bx < NB; ++bx)
            tma_load_2d_plain(sm.v[s][bx], &vmap, kcol + 64 * bx, krow + t * kT, &sm.v_full[s]);
        }
      }
      // every copy issued has landed before the CTA's shared memory can be released
      if (k > 0) mbar_wait(&sm.q_full, (k - 1) & 1, err);
      for (int t = g > 2 ? g - 2 : 0; t < g; ++t) {
        mbar_wait(&sm.k_full[t & 1], (t >> 1) & 1, err);
        mbar_wait(&sm.v_full[t & 1], (t >> 1) & 1, err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_qk = idesc_f16(kT, kT);
      constexpr uint32_t id_pv = idesc_f16(kT, HD, false, true);  // V: MN-major (hd contiguous)
      constexpr uint64_t kBoxD = kBox >> 4;                        // one box in the 16-byte address field
      const uint64_t dq = sw128_desc(smem_u32(sm.q[0])), dk0 = sw128_desc(smem_u32(sm.k[0][0]));
      const uint64_t dv0 = sw128_mn_desc(smem_u32(sm.v[0][0]), kBox);
      // S cursor (two tiles ahead of the PV cursor): item, tile in item, global tile, item count
      int qi = i0, qj = 0, qg = 0, qk_n = 0, qn = qi < items ? item_of(Pp, qi).n : 0;
      auto issue_s = [&]() {
        const int s = qg & 1;
        if (qj == 0) mbar_wait_ab(&sm.q_full, qk_n & 1, err, abort_s);
        mbar_wait_ab(&sm.k_full[s], (qg >> 1) & 1, err, abort_s);
        tc_fence_after();
        const uint64_t dk = dk0 + NB * s * kBoxD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)  // +32 bytes per K=16 step inside a 128-byte row
          umma_f16(tmem + kT * s, dq + (kk >> 2) * kBoxD + 2 * (kk & 3), dk + (kk >> 2) * kBoxD + 2 * (kk & 3), id_qk,
                   kk != 0);
        umma_commit(&sm.k_empty[s]);
        umma_commit(&sm.s_full[s]);
        ++qg;
        if (++qj == qn) {  // the item's last S MMA: its Q buffer frees when this completes
          umma_commit(&sm.q_empty);
          qj = 0;
          ++qk_n;
          qi += istep;
          qn = qi < items ? item_of(Pp, qi).n : 0;
        }
      };
      if (qn > 0) issue_s();
      if (qn > 0) issue_s();
      int pg = 0;
      for (int i = i0; i < items; i += istep) {
        const int n = item_of(Pp, i).n;
        for (int j = 0; j < n; ++j, ++pg) {
          const int s = pg & 1;
          mbar_wait_ab(&sm.p_full, pg & 1, err, abort_s);
          mbar_wait_ab(&sm.v_full[s], (pg >> 1) & 1, err, abort_s);
          tc_fence_after();
          const uint64_t dv = dv0 + NB * s * kBoxD;
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)  // 16 cache positions = 16 V rows of 128 bytes per step
            umma_f16_ts(tmem + kOCol, tmem + kPCol + 8 * kk, dv + kk * (2048 >> 4), id_pv, (j | kk) != 0);
          umma_commit(&sm.v_empty[s]);
          umma_commit(&sm.pv_done);
          if (qn > 0) issue_s();
        }
      }
      umma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, err);  // every MMA of this CTA has completed
    }
  } else {
    // ------------------------------------------------------------ softmax, then epilogue
    const int q4 = warp & 3;            // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // key columns 64*half .. +63 / head dims CW*half .. +CW-1
    const int r = 32 * q4 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q4) << 16) + 64 * half;    // its S columns
    const uint32_t orow = tmem + (static_cast<uint32_t>(32 * q4) << 16) + kOCol + CW * half;  // its O columns
    const float sl2 = Pp.scale_log2;
    // this thread's staging row: hd 128, its own buffer (64 head dims = 8 chunks); hd 64, the
    // row's 64 head dims in one buffer, this half's 32 at chunks 4*half ..
    constexpr int kSb = NB == 2 ? 1 : 0;
    uint8_t* const prow = sm.p[kSb * half] + r * 128;
    const int cbase = NB == 2 ? 0 : 4 * half;
    const uint32_t tp = tmem + (static_cast<uint32_t>(32 * q4) << 16) + kPCol + 32 * half;  // its P columns
    int g = 0;
    for (int i = i0; i < items; i += istep) {
      const Item it = item_of(Pp, i);
      float m = -INFINITY, l = 0.f;  // l: this half's partial row sum
      for (int j = 0; j < it.n; ++j, ++g) {
        const int s = g & 1;
        mbar_wait_ab(&sm.s_full[s], (g >> 1) & 1, err, abort_s);
        tc_fence_after();
        uint32_t raw[64];
        tmem_ld32_nowait(trow + kT * s, raw);
        tmem_ld32_nowait(trow + kT * s + 32, raw + 32);
        tmem_wait_ld();
        float x[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = __uint_as_float(raw[c]);
        if (Pp.causal ? j == it.qt : (j == it.n - 1 && (j + 1) * kT > P)) {
          // causal diagonal tile: keys after the query; non-causal last tile: keys at or past P
          const int lim = Pp.causal ? r - 64 * half : P - 1 - j * kT - 64 * half;  // columns c > lim masked
#pragma unroll
          for (int c = 0; c < 64; ++c) x[c] = c > lim ? -INFINITY : x[c];
        }
        float mk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mk[e] = x[e];
#pragma unroll
        for (int c = 8; c < 64; ++c) mk[c & 7] = fmaxf(mk[c & 7], x[c]);
        const float mpart = fmaxf(fmaxf(fmaxf(mk[0], mk[1]), fmaxf(mk[2], mk[3])),
                                  fmaxf(fmaxf(mk[4], mk[5]), fmaxf(mk[6], mk[7])));
        sm.xch[s][half][r] = mpart;
        named_bar(1 + q4, 64);  // the two warps of this lane quarter
        // the same max in both halves: max of the two partial maxima in a fixed order
        const float mx = fmaxf(sm.xch[s][0][r], sm.xch[s][1][r]) * sl2;
        float alpha = 1.f;
        if (mx > m + kRescale) {  // also the first tile (m = -inf): alpha = 0
          alpha = ex2(m - mx);
          m = mx;
        }
        float sk[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          x[c] = ex2(fmaf(x[c], sl2, -m));
          sk[c & 7] += x[c];
        }
        l = l * alpha + (((sk[0] + sk[1]) + (sk[2] + sk[3])) + ((sk[4] + sk[5]) + (sk[6] + sk[7])));
        if (j > 0) {
          // PV of the item's previous tile done: the P tile is free and O holds tiles 0 .. j-1
          // (at j == 0 the previous item's epilogue already waited for its last PV)
          mbar_wait_ab(&sm.pv_done, (g - 1) & 1, err, abort_s);
          tc_fence_after();
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
            for (int c = 0; c < CW; c += 32) {
              uint32_t o[32];
              tmem_ld32_nowait(orow + c, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(orow + c, o);
            }
            tmem_wait_st();
          }
        }
        {  // P row r, keys 64*half .. +63, as fp16 pairs into TMEM (the A operand of PV)
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) pk[e] = pack_h2(x[2 * e], x[2 * e + 1]);
          tmem_st32(tp, pk);
          tmem_wait_st();
        }
        if (j == it.n - 1 && (j + 1) * kT > P) {
          // key rows P .. of the item's last tile: their probabilities are 0, but 0 times a
          // non-finite value there would not be, so zero those V rows (whole 128-byte rows)
          mbar_wait_ab(&sm.v_full[s], (g >> 1) & 1, err, abort_s);
          const int nv = P - j * kT, nz = kT - nv;
          for (int e = tid - 64; e < NB * nz * 8; e += 32 * kSoftW) {
            const int box = e / (nz * 8), rem = e % (nz * 8);
            *reinterpret_cast<uint4*>(sm.v[s][box] + (nv + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full);
      }
      // ---- epilogue: O / l -> fp16 rows qt*128 + r, head dims CW*half .. +CW-1
      sm.xl[half][r] = l;
      named_bar(1 + q4, 64);
      const float lt = sm.xl[0][r] + sm.xl[1][r];
      mbar_wait_ab(&sm.pv_done, (g - 1) & 1, err, abort_s);  // the item's last PV: O complete, P tile free
      tc_fence_after();
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t o[32];
        tmem_ld32_nowait(orow + c, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // 16-byte chunk (cbase + c / 8 + e) of the staging row
          const float* f = reinterpret_cast<const float*>(o + 8 * e);
          const int ch = cbase + c / 8 + e;
          *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) =
              make_uint4(pack_h2(f[0] * inv, f[1] * inv), pack_h2(f[2] * inv, f[3] * inv),
                         pack_h2(f[4] * inv, f[5] * inv), pack_h2(f[6] * inv, f[7] * inv));
        }
      }
      __syncwarp();  // this warp's 32 rows x CW columns are staged; write them as row segments
      // (hd 128: chunk ch of head dims 64*half ..; hd 64: chunk ch of the head's 64 dims)
      __half* const obase = Pp.o + (int64_t)it.h * HD + (NB == 2 ? 64 * half : 0);
      constexpr int kCh = CW / 8;  // 16-byte chunks per row of this warp
#pragma unroll
      for (int e = 0; e < kCh; ++e) {
        const int rr = 32 * q4 + (32 / kCh) * e + lane / kCh, ch = cbase + lane % kCh;  // row, 16-byte chunk
        const int pos = it.qt * kT + rr;
        const uint4 v = *reinterpret_cast<const uint4*>(sm.p[kSb * half] + rr * 128 + ((ch ^ (rr & 7)) << 4));
        if (pos < P) *reinterpret_cast<uint4*>(obase + ((int64_t)it.b * P + pos) * Pp.ldo + 8 * ch) = v;
      }
      __syncwarp();  // reads of the staging rows done before this warp writes the next item's P
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// [rows, cols] fp16 (row stride ld elements), 64-column x 128-row boxes, 128B swizzle
bool fa_map(const void* base, int64_t rows, int64_t cols, int64_t ld, CUtensorMap* out) {
  struct Key {
    const void* p;
    int64_t rows, cols, ld;
    bool operator==(const Key& o) const { return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ (std::hash<int64_t>()(k.rows) * 31) ^ (std::hash<int64_t>()(k.ld) * 17);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  const Key key{base, rows, cols, ld};
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
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kT)};
  cuuint32_t es[2] = {1, 1};
  if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

template <int HD>
int launch_attn(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const FaParams& p,
                hm_stream_t stream) {
  const size_t smem = sizeof(FaSmem<HD / 64>) + 1024;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms < 1)
    return HM_EARG;
  const unsigned ctas = static_cast<unsigned>(p.items < sms ? p.items : sms);  // persistent: one CTA per SM
  const cudaError_t e =
      hm_launch(prefill_attn_tc_kernel<HD>, dim3(ctas), dim3(kThreads), smem, stream, false, qm, km, vm, p);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

}  // namespace

extern "C" int hm_prefill_attn(const void* q, const void* kc, const void* vc, void* o, int B, int P, int Hq, int Hk,
                               int hd, int L, float scale, int* err, hm_stream_t stream) {
  if (!q || !kc || !vc || !o || B < 1 || P < 1 || Hk < 1 || Hq < Hk || Hq % Hk != 0 || hd != 128 || P > L)
    return HM_EARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(kc) |
       reinterpret_cast<uintptr_t>(vc)) & 15u)
    return HM_EARG;
  const int64_t kv_rows = (int64_t)B * Hk * L, q_rows = (int64_t)B * P;
  const int64_t nqt = (P + kT - 1) / kT, items = nqt * Hq * B;
  if (kv_rows + kT > INT32_MAX || q_rows + kT > INT32_MAX || items > INT32_MAX) return HM_EARG;
  CUtensorMap qm, km, vm;
  if (!fa_map(q, q_rows, (int64_t)Hq * hd, (int64_t)Hq * hd, &qm) || !fa_map(kc, kv_rows, hd, hd, &km) ||
      !fa_map(vc, kv_rows, hd, hd, &vm))
    return HM_EARG;
  FaParams p;
  p.o = reinterpret_cast<__half*>(o);
  p.ldo = (int64_t)Hq * hd;
  p.B = B;
  p.P = P;
  p.Hq = Hq;
  p.Hk = Hk;
  p.L = L;
  p.items = static_cast<int>(items);
  p.causal = 1;
  p.kv_b_rows = Hk * L;
  p.kv_h_rows = L;
  p.kv_h_cols = 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  return launch_attn<128>(qm, km, vm, p, stream);
}

extern "C" int hm_codec_attn(const void* q, const void* k, const void* v, void* o, int B, int T, int H, int hd,
                             int64_t ld, int64_t ldo, float scale, int* err, hm_stream_t stream) {
  if (!q || !k || !v || !o || B < 1 || T < 1 || H < 1 || (hd != 64 && hd != 128)) return HM_EARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) & 15u)
    return HM_EARG;
  if (ld < (int64_t)H * hd || ld % 8 || ldo < (int64_t)H * hd || ldo % 8) return HM_EARG;
  const int64_t rows = (int64_t)B * T, nqt = (T + kT - 1) / kT, items = nqt * H * B;
  if (rows + kT > INT32_MAX || items > INT32_MAX) return HM_EARG;
  CUtensorMap qm, km, vm;
  if (!fa_map(q, rows, (int64_t)H * hd, ld, &qm) || !fa_map(k, rows, (int64_t)H * hd, ld, &km) ||
      !fa_map(v, rows, (int64_t)H * hd, ld, &vm))
    return HM_EARG;
  FaParams p;
  p.o = reinterpret_cast<__half*>(o);
  p.ldo = ldo;
  p.B = B;
  p.P = T;
  p.Hq = H;
  p.Hk = H;
  p.L = T;
  p.items = static_cast<int>(items);
  p.causal = 0;
  p.kv_b_rows = T;
  p.kv_h_rows = 0;
  p.kv_h_cols = hd;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  return hd == 64 ? launch_attn<64>(qm, km, vm, p, stream) : launch_attn<128>(qm, km, vm, p, stream);
}
