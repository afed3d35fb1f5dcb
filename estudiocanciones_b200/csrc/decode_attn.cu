// Split-K GQA decode attention over the static KV cache (sm_100a).
//
// Replaces `_attn` + `_attn_combine` (app/kernels.py:112-167) as launched by
// Stack.decode (app/engine.py:194-204).  Row r (batch r / S) attends to cache
// positions [0, pos[r]], read from device memory so one CUDA graph serves every
// frame.  The G = Hq/Hk query heads of a KV head share one pass over its K/V
// (no KV copy per group).
//
// Grid (nsplit, Hk, R), 128 threads.  Each CTA streams its position range in
// tiles of 32 positions; the K and V rows of a tile are contiguous in the cache
// ([B, Hk, L, hd] layout), so each tile is two 1-D bulk copies into a
// double-buffered shared-memory ring completed on mbarriers.  Scores and the
// PV product run in fp32 on CUDA cores (the kernel is HBM-bound: 2*G*hd FMAs
// per 4*hd bytes); probabilities are rounded to fp16 before the PV product
// and the normaliser keeps the fp32 sum, as in _attn.  With nsplit > 1 the
// last CTA of each (row, KV head) merges the split partials (log-sum-exp) and
// re-arms its ticket.
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "hm_common.cuh"

namespace {

constexpr int kTP = 32;       // positions per tile
constexpr int kThreads = 128;
constexpr int kMaxG = 8;

struct AttnParams {
  const __half* q;
  const __half* kc;
  const __half* vc;
  const int64_t* pos;
  __half* o;
  int R, S, Hq, Hk, L, nsplit;
  float scale;
  float* ws;
  int* counters;
  int* err;
  int cluster;  // tensor-core kernel: the nsplit CTAs of a (row, KV head) form a cluster and merge in DSMEM
  int box3;     // tensor-core kernel: K / V maps are 3-D, one request per tile of each (else two 2-D boxes)
};

constexpr int kMaxSplit = 64;

template <int HD>
struct AttnCfg {
  static constexpr int NST = HD <= 128 ? 4 : 2;  // K/V ring stages (16 KB each at hd 128)
};

template <int HD>
struct AttnSmem {
  __half k[AttnCfg<HD>::NST][kTP][HD];
  __half v[AttnCfg<HD>::NST][kTP][HD];
  float q[kMaxG][HD];
  float s[kMaxG][kTP];
  float red[kMaxG][HD];
  float alpha[kMaxG], m[kMaxG], l[kMaxG];
  float cw[kMaxG][kMaxSplit];  // combine weights of the split partials
  float cl[kMaxG][kMaxSplit];  // their softmax denominators
  float cden[kMaxG];
  uint64_t bar[AttnCfg<HD>::NST];
  int flag;
  int abort_flag;
};

template <int HD>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const __grid_constant__ AttnParams P) {
  constexpr int CPT = HD / 32;  // 16-byte chunks of a K row per thread (4 threads per position)
  constexpr int U = HD / 128;   // half2 columns per thread in the PV product
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<HD>& sm = *reinterpret_cast<AttnSmem<HD>*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = blockIdx.x, kh = blockIdx.y, r = blockIdx.z;
  // parameters in registers: the waits and barriers below clobber memory, which would
  // otherwise re-read every field from the parameter block inside the loops
  const int Hq = P.Hq, Hk = P.Hk, S = P.S, L = P.L, nsplit = P.nsplit, R = P.R;
  const float scale = P.scale;
  int* const err = P.err;
  const __half* const qg = P.q;
  __half* const og = P.o;
  float* const wsg = P.ws;
  int* const counters = P.counters;
  const int G = Hq / Hk;

  constexpr int NST = AttnCfg<HD>::NST;
  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < NST; ++i) mbar_init(&sm.bar[i], 1);
    fence_barrier_init();
  }
  pdl_trigger();
  pdl_wait();

  const int64_t p_last = P.pos[r];
  const int b = r / S;
  int len = static_cast<int>(p_last) + 1;
  if (p_last < 0 || p_last >= L) {
    report_error(err, HM_ERR_BADINDEX);
    len = 0;
  }
  const int per = (len + nsplit - 1) / nsplit;
  const int chunk = (per + kTP - 1) / kTP * kTP;
  const int lo = sp * chunk;
  const int hi = min(len, lo + chunk);
  const int ntile = hi > lo ? (hi - lo + kTP - 1) / kTP : 0;

  const __half* kbase = P.kc + ((int64_t)b * Hk + kh) * L * HD;
  const __half* vbase = P.vc + ((int64_t)b * Hk + kh) * L * HD;

  // q of the G heads of this KV head, fp32 (16-byte loads, all in flight together)
  for (int i = tid; i < G * HD / 8; i += kThreads) {
    const int gg = (8 * i) / HD, d = 8 * i - gg * HD;
    const uint4 v = *reinterpret_cast<const uint4*>(qg + (int64_t)r * Hq * HD + (kh * G + gg) * HD + d);
    const __half2* h2 = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h2[j]);
      sm.q[gg][d + 2 * j] = f.x;
      sm.q[gg][d + 2 * j + 1] = f.y;
    }
  }
  if (tid < kMaxG) {
    sm.m[tid] = -INFINITY;
    sm.l[tid] = 0.f;
  }
  __syncthreads();

  auto issue = [&](int t) {
    const int st = t % NST;
    const int p0 = lo + t * kTP;
    const int nv = min(kTP, hi - p0);
    const uint32_t bytes = static_cast<uint32_t>(nv) * HD * 2;
    mbar_arrive_expect_tx(&sm.bar[st], 2 * bytes);
    bulk_load(&sm.k[st][0][0], kbase + (int64_t)p0 * HD, bytes, &sm.bar[st]);
    bulk_load(&sm.v[st][0][0], vbase + (int64_t)p0 * HD, bytes, &sm.bar[st]);
  };
  if (tid == 0)
    for (int t = 0; t < NST && t < ntile; ++t) issue(t);

  float acc[kMaxG][2 * U];
#pragma unroll
  for (int gg = 0; gg < kMaxG; ++gg)
#pragma unroll
    for (int u = 0; u < 2 * U; ++u) acc[gg][u] = 0.f;

  const int qp = tid >> 2, qd = tid & 3;   // QK: position qp of the tile, quarter qd of the row
  const int ph = tid >> 6, dc = tid & 63;  // PV: position parity ph, half2 column group dc
  for (int t = 0; t < ntile; ++t) {
    const int st = t % NST;
    const int p0 = lo + t * kTP;
    const int nv = min(kTP, hi - p0);
    mbar_wait_ab(&sm.bar[st], (t / NST) & 1, err, &sm.abort_flag);  // on timeout: carry on, error flagged
    // ---- scores s[g][p] = (q_g . k_p) * scale
    {
      float part[kMaxG];
#pragma unroll
      for (int gg = 0; gg < kMaxG; ++gg) part[gg] = 0.f;
      if (qp < nv) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
          const int c = qd * CPT + (i + qd + (qp & 1)) % CPT;   // rotated chunk order (bank spread)
          const uint4 kv = *reinterpret_cast<const uint4*>(&sm.k[st][qp][c * 8]);
          const __half2* kh2 = reinterpret_cast<const __half2*>(&kv);
          float kf[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(kh2[j]);
            kf[2 * j] = f.x;
            kf[2 * j + 1] = f.y;
          }
#pragma unroll
          for (int gg = 0; gg < kMaxG; ++gg) {
            if (gg < G) {
              const float4 q0 = *reinterpret_cast<const float4*>(&sm.q[gg][c * 8]);
              const float4 q1 = *reinterpret_cast<const float4*>(&sm.q[gg][c * 8 + 4]);
              part[gg] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] +
                          q1.y * kf[5] + q1.z * kf[6] + q1.w * kf[7];
            }
          }
        }
      }
#pragma unroll
      for (int gg = 0; gg < kMaxG; ++gg) {
        float v = part[gg];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (gg < G && qd == 0) sm.s[gg][qp] = qp < nv ? v * scale : -INFINITY;
      }
    }
    __syncthreads();
    // ---- online softmax update per head (lane = position)
    for (int gg = warp; gg < G; gg += kThreads / 32) {
      const float sc = sm.s[gg][lane];
      const float m_old = sm.m[gg];
      const float m_new = fmaxf(m_old, warp_max(sc));
      float pe = 0.f, alpha = 1.f;
      if (m_new != -INFINITY) {
        pe = sc == -INFINITY ? 0.f : expf(sc - m_new);
        alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
      }
      const float tot = warp_sum(pe);
      sm.s[gg][lane] = __half2float(__float2half_rn(pe));
      if (lane == 0) {
        sm.alpha[gg] = alpha;
        sm.m[gg] = m_new;
        sm.l[gg] = sm.l[gg] * alpha + tot;
      }
    }
    __syncthreads();
    // ---- acc = acc*alpha + P V
#pragma unroll
    for (int gg = 0; gg < kMaxG; ++gg) {
      if (gg < G) {
        const float a = sm.alpha[gg];
#pragma unroll
        for (int u = 0; u < 2 * U; ++u) acc[gg][u] *= a;
      }
    }
    for (int p = ph; p < nv; p += 2) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float2 vf = __half22float2(*reinterpret_cast<const __half2*>(&sm.v[st][p][2 * (dc + 64 * u)]));
#pragma unroll
        for (int gg = 0; gg < kMaxG; ++gg) {
          if (gg < G) {
            const float pr = sm.s[gg][p];
            acc[gg][2 * u] += pr * vf.x;
            acc[gg][2 * u + 1] += pr * vf.y;
          }
        }
      }
    }
    __syncthreads();  // stage st and s[][] are free again
    if (tid == 0 && t + NST < ntile) issue(t + NST);
  }

  // ---- merge the two position parities into red[g][d]
  if (ph == 1) {
#pragma unroll
    for (int gg = 0; gg < kMaxG; ++gg)
      if (gg < G)
#pragma unroll
        for (int u = 0; u < U; ++u) {
          sm.red[gg][2 * (dc + 64 * u)] = acc[gg][2 * u];
          sm.red[gg][2 * (dc + 64 * u) + 1] = acc[gg][2 * u + 1];
        }
  }
  __syncthreads();
  if (ph == 0) {
#pragma unroll
    for (int gg = 0; gg < kMaxG; ++gg)
      if (gg < G)
#pragma unroll
        for (int u = 0; u < U; ++u) {
          sm.red[gg][2 * (dc + 64 * u)] += acc[gg][2 * u];
          sm.red[gg][2 * (dc + 64 * u) + 1] += acc[gg][2 * u + 1];
        }
  }
  __syncthreads();

  const int64_t head0 = (int64_t)r * Hq + kh * G;
  if (nsplit == 1) {
    for (int i = tid; i < G * HD; i += kThreads) {
      const int gg = i / HD, d = i - gg * HD;
      const float l = sm.l[gg];
      og[(head0 + gg) * HD + d] = __float2half_rn(l > 0.f ? sm.red[gg][d] / l : 0.f);
    }
    return;
  }
  const int64_t nh = (int64_t)R * Hq * nsplit;
  float* wm = wsg;
  float* wl = wsg + nh;
  float* wa = wsg + 2 * nh;
  for (int i = tid; i < G * HD; i += kThreads) {
    const int gg = i / HD, d = i - gg * HD;
    wa[((head0 + gg) * nsplit + sp) * HD + d] = sm.red[gg][d];
  }
  if (tid < G) {
    wm[(head0 + tid) * nsplit + sp] = sm.m[tid];
    wl[(head0 + tid) * nsplit + sp] = sm.l[tid];
  }
  __threadfence();
  __syncthreads();
  int* ticket = &counters[r * Hk + kh];
  if (tid == 0) sm.flag = (atomicAdd(ticket, 1) == nsplit - 1);
  __syncthreads();
  if (!sm.flag) return;
  __threadfence();
  // merge the nsplit partials of the G heads: weights exp(m_s - max) staged first (one
  // load per thread), then every output sums its column over the splits in order
  for (int i = tid; i < G * nsplit; i += kThreads) {
    const int gg = i / nsplit, s2 = i - gg * nsplit;
    sm.cw[gg][s2] = __ldcg(wm + (head0 + gg) * nsplit + s2);
    sm.cl[gg][s2] = __ldcg(wl + (head0 + gg) * nsplit + s2);
  }
  __syncthreads();
  if (tid < G) {
    float mx = -INFINITY;
    for (int s2 = 0; s2 < nsplit; ++s2) mx = fmaxf(mx, sm.cw[tid][s2]);
    float den = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2) {
      const float ms = sm.cw[tid][s2];
      const float w = ms > -INFINITY ? expf(ms - mx) : 0.f;
      sm.cw[tid][s2] = w;
      den += sm.cl[tid][s2] * w;
    }
    sm.cden[tid] = den;
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += kThreads) {
    const int gg = i / HD, d = i - gg * HD;
    const int64_t h = head0 + gg;
    float part[8];
    float num = 0.f;
    for (int s0 = 0; s0 < nsplit; s0 += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        part[j] = s0 + j < nsplit ? __ldcg(wa + (h * nsplit + s0 + j) * HD + d) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < nsplit) num += part[j] * sm.cw[gg][s0 + j];
    }
    const float den = sm.cden[gg];
    og[h * HD + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) *ticket = 0;
}

// ------------------------------------------------------------------ tensor-core path (hd = 128)
// Same contract as decode_attn_kernel for head_dim 128, with QK^T and PV on the
// tensor cores (FA2-style): the G query heads of the KV head are the rows of a
// 16-row MMA tile (rows >= G are zero), each warp owns 16 positions of every
// 64-position stage, scores stay in registers, probabilities are rounded to fp16
// and fed straight back as the A operand of the PV MMA.  K and V tiles arrive by
// 2-D TMA (box 64 dims x 64 positions, 128B swizzle) through a 3-stage ring.
constexpr int kTcPos = 64;   // positions per stage (4 warps x 16)
constexpr int kTcNst = 3;
constexpr int kTcBox = kTcPos * 128;  // bytes of one 64x64 fp16 box
constexpr int kMaxCluster = 4;        // splits merged inside a cluster
constexpr int kMaxPushG = 4;          // query heads per KV head of the cluster merge

struct TcSmem {
  uint8_t k[kTcNst][2][kTcBox];  // [stage][dims 0-63 | 64-127][64 positions x 128 B]
  uint8_t v[kTcNst][2][kTcBox];
  float mw[4][kMaxG], lw[4][kMaxG];
  float cw[kMaxG][kMaxSplit], cl[kMaxG][kMaxSplit], cden[kMaxG];
  float cm[kMaxG], cd[kMaxG];  // this CTA's split maxima and denominators (cluster merge)
  // cluster merge, rank 0 only: the partials the other splits push (num, maxima, denominators)
  float cpush[kMaxCluster - 1][kMaxPushG][128];
  float cpm[kMaxCluster - 1][kMaxPushG], cpl[kMaxCluster - 1][kMaxPushG];
  float fw[4][kMaxG], hm[kMaxG], hd[kMaxG];  // per head: warp weights, maximum, denominator
  uint64_t bar[kTcNst];
  uint64_t cready;  // cluster merge: the partials of every other split are in rank 0's shared memory
  int flag, abort_flag;
};

__device__ __forceinline__ uint32_t swz(const uint8_t* box, int row, int chunk) {
  return smem_u32(box + row * 128 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kThreads) decode_attn_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                  const __grid_constant__ CUtensorMap vmap,
                                                                  const __grid_constant__ AttnParams P) {
  constexpr int HD = 128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int sp = blockIdx.x, kh = blockIdx.y, r = blockIdx.z;
  const int Hq = P.Hq, Hk = P.Hk, S = P.S, L = P.L, nsplit = P.nsplit, R = P.R;
  const float scale = P.scale;
  int* const err = P.err;
  __half* const og = P.o;
  float* const wsg = P.ws;
  int* const counters = P.counters;
  const int G = Hq / Hk;

  const bool clus = P.cluster != 0 && nsplit > 1;
  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < kTcNst; ++i) mbar_init(&sm.bar[i], 1);
    if (clus) mbar_init(&sm.cready, nsplit - 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (clus) cluster_sync_all();  // every CTA's merge barriers exist before any remote arrival
  if (smem_u32(smem_raw) & 1023u) {  // (the same for every CTA: all return)
    if (tid == 0) report_error(err, HM_ERR_TIMEOUT);
    return;
  }
  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  pdl_trigger();

  // Positions come from a buffer no launch of the frame writes (the frame commit, a
  // graph replay earlier, advances them), and cache slots before pos[r] were written by
  // earlier steps: the first K/V tiles that end before pos[r] are fetched before
  // griddepcontrol.wait, overlapping the tail of the producing qkv launch.  The tile
  // holding pos[r] (written by that launch) is fetched after the wait.
  const int64_t p_last = P.pos[r];
  const int b = r / S;
  int len = static_cast<int>(p_last) + 1;
  if (p_last < 0 || p_last >= L) {
    report_error(err, HM_ERR_BADINDEX);
    len = 0;
  }
  const int per = (len + nsplit - 1) / nsplit;
  const int chunk = (per + kTcPos - 1) / kTcPos * kTcPos;
  const int lo = sp * chunk;
  const int hi = min(len, lo + chunk);
  const int ntile = hi > lo ? (hi - lo + kTcPos - 1) / kTcPos : 0;
  const int row0 = ((b * Hk + kh) * L) + lo;

  auto issue = [&](int tt) {
    const int st = tt % kTcNst;
    const int y = row0 + tt * kTcPos;
    mbar_arrive_expect_tx(&sm.bar[st], 4 * kTcBox);
    if (P.box3) {  // both 64-dim halves of the tile in one request each for K and V
      tma_load_3d_plain(sm.k[st][0], &kmap, 0, y, 0, &sm.bar[st]);
      tma_load_3d_plain(sm.v[st][0], &vmap, 0, y, 0, &sm.bar[st]);
    } else {
      tma_load_2d_plain(sm.k[st][0], &kmap, 0, y, &sm.bar[st]);
      tma_load_2d_plain(sm.k[st][1], &kmap, 64, y, &sm.bar[st]);
      tma_load_2d_plain(sm.v[st][0], &vmap, 0, y, &sm.bar[st]);
      tma_load_2d_plain(sm.v[st][1], &vmap, 64, y, &sm.bar[st]);
    }
  };
  const int n_first = min(kTcNst, ntile);
  int n_early = 0;  // leading tiles that end before pos[r]
  while (n_early < n_first && lo + (n_early + 1) * kTcPos <= static_cast<int>(p_last)) ++n_early;
  if (tid == 0)
    for (int tt = 0; tt < n_early; ++tt) issue(tt);
  pdl_wait();
  if (tid == 0) {
    fence_proxy_async_global();  // the qkv launch's cache writes, before the TMA reads them
    for (int tt = n_early; tt < n_first; ++tt) issue(tt);
  }

  // q of this lane's head (row g of the MMA tile), as A fragments for 8 k-steps
  uint32_t qa[8][2];
  {
    const __half* qh = P.q + ((int64_t)r * Hq + kh * G + g) * HD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + 16 * ks + 2 * t) : 0u;
      qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + 16 * ks + 8 + 2 * t) : 0u;
    }
  }
  float m_run = -INFINITY, l_run = 0.f;
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int mi = lane >> 3, ri = lane & 7;

  for (int tt = 0; tt < ntile; ++tt) {
    const int st = tt % kTcNst;
    mbar_wait_ab(&sm.bar[st], (tt / kTcNst) & 1, err, &sm.abort_flag);  // on timeout: carry on, error flagged
    const int nvalid = min(16, hi - (lo + tt * kTcPos + warp * 16));
    if (nvalid > 0) {
      // ---- S = Q K^T over this warp's 16 positions (two n-tiles of 8)
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const int kp = warp * 16 + (mi >= 2 ? 8 : 0) + ri;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int c = 2 * ks + (mi & 1);
        uint32_t b00, b01, b10, b11;
        ldsm_x4(b00, b01, b10, b11, swz(sm.k[st][c >> 3], kp, c & 7));
        mma_16816(s[0], qa[ks][0], 0u, qa[ks][1], 0u, b00, b01);
        mma_16816(s[1], qa[ks][0], 0u, qa[ks][1], 0u, b10, b11);
      }
      // ---- online softmax for head g (the quad t = 0..3 holds its 16 scores)
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
      // ---- acc += fp16(P) V
      const uint32_t pa0 = pack_h2(pv[0], pv[1]), pa2 = pack_h2(pv[2], pv[3]);
      const int vp = warp * 16 + (mi & 1) * 8 + ri;
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        const int c = 2 * nd + (mi >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(v0, v1, v2, v3, swz(sm.v[st][c >> 3], vp, c & 7));
        mma_16816(acc[2 * nd], pa0, 0u, pa2, 0u, v0, v1);
        mma_16816(acc[2 * nd + 1], pa0, 0u, pa2, 0u, v2, v3);
      }
    }
    __syncthreads();  // every warp is done with stage st
    if (tid == 0 && tt + kTcNst < ntile) issue(tt + kTcNst);
  }

  // ---- merge the four warps (red aliases the now idle stage-0 K buffers)
  float* red = reinterpret_cast<float*>(&sm.k[0][0][0]);  // [4][kMaxG][128]
  float* cnum = reinterpret_cast<float*>(&sm.k[1][0][0]);  // [G][128] this split's partial (cluster merge)
  if (g < G) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      red[(warp * kMaxG + g) * HD + 8 * i + 2 * t] = acc[i][0];
      red[(warp * kMaxG + g) * HD + 8 * i + 2 * t + 1] = acc[i][1];
    }
    if (t == 0) {
      sm.mw[warp][g] = m_run;
      sm.lw[warp][g] = l_run;
    }
  }
  __syncthreads();
  // per head (once, not per element): the warps' maximum, weights and denominator
  if (tid < G) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm.mw[w][tid]);
    float den = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sm.mw[w][tid];
      const float f = mw > -INFINITY ? expf(mw - M) : 0.f;
      sm.fw[w][tid] = f;
      den += sm.lw[w][tid] * f;
    }
    sm.hm[tid] = M;
    sm.hd[tid] = den;
  }
  __syncthreads();
  const int64_t head0 = (int64_t)r * Hq + kh * G;
  const int64_t nh = (int64_t)R * Hq * nsplit;
  float* wm = wsg;
  float* wl = wsg + nh;
  float* wa = wsg + 2 * nh;
  for (int i = tid; i < G * HD; i += kThreads) {
    const int gg = i / HD, d = i - gg * HD;
    const float M = sm.hm[gg], den = sm.hd[gg];
    float num = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) num += red[(w * kMaxG + gg) * HD + d] * sm.fw[w][gg];
    if (nsplit == 1) {
      og[(head0 + gg) * HD + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
    } else if (clus) {
      const uint32_t rank = cluster_ctarank();
      if (rank == 0) {
        cnum[gg * HD + d] = num;
      } else {  // straight into rank 0's shared memory
        st_dsmem_f32(dsmem_addr(&sm.cpush[rank - 1][gg][d], 0), num);
        if (d == 0) {
          st_dsmem_f32(dsmem_addr(&sm.cpm[rank - 1][gg], 0), M);
          st_dsmem_f32(dsmem_addr(&sm.cpl[rank - 1][gg], 0), den);
        }
      }
    } else {
      wa[((head0 + gg) * nsplit + sp) * HD + d] = num;
      if (d == 0) {
        wm[(head0 + gg) * nsplit + sp] = M;
        wl[(head0 + gg) * nsplit + sp] = den;
      }
    }
  }
  if (nsplit == 1) return;
  if (clus) {
    // ---- split merge inside the cluster: the other splits have pushed their partials
    // into rank 0's shared memory; they signal rank 0 and exit (nothing reads their own
    // shared memory), rank 0 merges in split order (the same arithmetic as the workspace
    // path below) from local memory.
    __syncthreads();
    const uint32_t rank = cluster_ctarank();
    if (rank != 0) {
      if (tid == 0) {
        fence_acq_rel_cluster();
        mbar_arrive_dsmem(dsmem_addr(&sm.cready, 0));
      }
      return;
    }
    if (tid == 0) mbar_wait_cluster(&sm.cready, 0, err);
    __syncthreads();
    // per head (once): split maxima / denominators -> weights and the merged denominator
    if (tid < G) {
      float ms[kMaxCluster], ls[kMaxCluster];
#pragma unroll
      for (int s2 = 0; s2 < kMaxCluster; ++s2) {
        ms[s2] = s2 >= nsplit ? -INFINITY : (s2 == 0 ? sm.hm[tid] : sm.cpm[s2 - 1][tid]);
        ls[s2] = s2 >= nsplit ? 0.f : (s2 == 0 ? sm.hd[tid] : sm.cpl[s2 - 1][tid]);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int s2 = 0; s2 < kMaxCluster; ++s2)
        if (s2 < nsplit) mx = fmaxf(mx, ms[s2]);
      float den = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kMaxCluster; ++s2) {
        if (s2 < nsplit) {
          const float w = ms[s2] > -INFINITY ? expf(ms[s2] - mx) : 0.f;
          sm.cw[tid][s2] = w;
          den += ls[s2] * w;
        }
      }
      sm.cden[tid] = den;
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += kThreads) {
      const int gg = i / HD, d = i - gg * HD;
      float num = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kMaxCluster; ++s2)
        if (s2 < nsplit) num += (s2 == 0 ? cnum[i] : sm.cpush[s2 - 1][gg][d]) * sm.cw[gg][s2];
      const float den = sm.cden[gg];
      og[(head0 + gg) * HD + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
    }
    return;
  }
  __threadfence();
  __syncthreads();
  int* ticket = &counters[r * Hk + kh];
  if (tid == 0) sm.flag = (atomicAdd(ticket, 1) == nsplit - 1);
  __syncthreads();
  if (!sm.flag) return;
  __threadfence();
  for (int i = tid; i < G * nsplit; i += kThreads) {
    const int gg = i / nsplit, s2 = i - gg * nsplit;
    sm.cw[gg][s2] = __ldcg(wm + (head0 + gg) * nsplit + s2);
    sm.cl[gg][s2] = __ldcg(wl + (head0 + gg) * nsplit + s2);
  }
  __syncthreads();
  if (tid < G) {
    float mx = -INFINITY;
    for (int s2 = 0; s2 < nsplit; ++s2) mx = fmaxf(mx, sm.cw[tid][s2]);
    float den = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2) {
      const float ms = sm.cw[tid][s2];
      const float w = ms > -INFINITY ? expf(ms - mx) : 0.f;
      sm.cw[tid][s2] = w;
      den += sm.cl[tid][s2] * w;
    }
    sm.cden[tid] = den;
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += kThreads) {
    const int gg = i / HD, d = i - gg * HD;
    const int64_t h = head0 + gg;
    float part[8];
    float num = 0.f;
    for (int s0 = 0; s0 < nsplit; s0 += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) part[j] = s0 + j < nsplit ? __ldcg(wa + (h * nsplit + s0 + j) * HD + d) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < nsplit) num += part[j] * sm.cw[gg][s0 + j];
    }
    const float den = sm.cden[gg];
    og[h * HD + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) *ticket = 0;
}

// View of an fp16 cache [rows = B*Hk*L, 128] for the TMA (cached by pointer and kind):
//  2-D {128, rows}, box 64 dims x 64 positions: two requests per tile;
//  3-D {64, rows, 2} (dim within a half, position, half; the half stride is 128 bytes),
//  box {64, 64, 2}: one request per tile, laid out in shared memory as [half][position][128 B],
//  the two 2-D boxes one after the other.
bool cache_map(const void* base, int64_t rows, bool three_d, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::pair<int64_t, CUtensorMap>> cache[2];
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache[three_d].find(base);
    if (it != cache[three_d].end() && it->second.first == rows) {
      *out = it->second.second;
      return true;
    }
  }
  auto enc = hm_encode_fn();
  if (!enc) return false;
  CUtensorMap m;
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r;
  if (three_d) {
    cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), 2};
    cuuint64_t strides[2] = {256, 128};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kTcPos), 2};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {256};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kTcPos)};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[three_d].size() > 4096) cache[three_d].clear();
  cache[three_d][base] = {rows, m};
  *out = m;
  return true;
}

int attn_box_on() {
  static const int on = [] {
    const char* e = getenv("HM_ATTN_BOX");
    return e ? atoi(e) : 1;
  }();
  return on;
}

// HM_ATTN_TC=0 selects the CUDA-core kernel for head_dim 128 (comparison runs)
bool attn_tc_enabled() {
  static const int on = [] {
    const char* e = getenv("HM_ATTN_TC");
    return e ? atoi(e) : 1;
  }();
  return on != 0;
}

cudaError_t launch_attn_tc(const AttnParams& p, int B, int pdl, cudaStream_t st) {
  const int64_t rows = (int64_t)B * p.Hk * p.L;
  // one request per K / V tile (HM_ATTN_BOX=1, the default), else two 2-D boxes each: the
  // same bytes land at the same shared-memory addresses either way
  CUtensorMap km, vm;
  bool three_d = attn_box_on() && cache_map(p.kc, rows, true, &km) && cache_map(p.vc, rows, true, &vm);
  if (!three_d && (!cache_map(p.kc, rows, false, &km) || !cache_map(p.vc, rows, false, &vm)))
    return cudaErrorInvalidValue;
  const size_t smem = sizeof(TcSmem) + 1024;  // + slack to align the base to 1024
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    hm_carveout(decode_attn_tc_kernel);
    configured = true;
  }
  // 2..8 splits: one cluster per (row, KV head), merged in DSMEM (no workspace round trip)
  static const int clus_on = [] {
    const char* e = getenv("HM_ATTN_CLUSTER");
    return e ? atoi(e) : 1;
  }();
  AttnParams q = p;
  q.box3 = three_d ? 1 : 0;
  q.cluster = clus_on && p.nsplit >= 2 && p.nsplit <= kMaxCluster && p.Hq / p.Hk <= kMaxPushG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nsplit, p.Hk, p.R);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (q.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = p.nsplit;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, decode_attn_tc_kernel, km, vm, q);
}

template <int HD>
cudaError_t launch_attn(const AttnParams& p, int pdl, cudaStream_t st) {
  const size_t smem = sizeof(AttnSmem<HD>);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return hm_launch(decode_attn_kernel<HD>, dim3(p.nsplit, p.Hk, p.R), dim3(kThreads), smem, st, pdl, p);
}

}  // namespace


extern "C" int hm_decode_attn_box_form(const void* cache, int64_t rows) {
  if (!cache || rows < 1 || (reinterpret_cast<uintptr_t>(cache) & 15u)) return HM_EARG;
  CUtensorMap m;
  if (attn_box_on() && cache_map(cache, rows, true, &m)) return 1;
  return cache_map(cache, rows, false, &m) ? 0 : HM_EARG;
}

extern "C" size_t hm_decode_attn_workspace_bytes(int R, int Hq, int hd, int nsplit) {
  if (nsplit <= 1) return 0;
  return static_cast<size_t>(R) * Hq * nsplit * (hd + 2) * sizeof(float);
}

extern "C" int hm_decode_attn(const void* q, const void* kc, const void* vc, const int64_t* pos, void* o, int R,
                              int S, int Hq, int Hk, int hd, int L, float scale, int nsplit, void* ws,
                              size_t ws_bytes, int* counters, int n_counters, int* err, int pdl,
                              hm_stream_t stream) {
  if (!q || !kc || !vc || !pos || !o || R < 1 || S < 1 || R % S || Hk < 1 || Hq % Hk || Hq / Hk > kMaxG || L < 1 ||
      nsplit < 1 || nsplit > kMaxSplit)
    return HM_EARG;
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15u) return HM_EARG;
  if (nsplit > 1 && (!ws || !counters || n_counters < R * Hk || ws_bytes < hm_decode_attn_workspace_bytes(R, Hq, hd, nsplit)))
    return HM_EARG;
  AttnParams p;
  p.q = reinterpret_cast<const __half*>(q);
  p.kc = reinterpret_cast<const __half*>(kc);
  p.vc = reinterpret_cast<const __half*>(vc);
  p.pos = pos;
  p.o = reinterpret_cast<__half*>(o);
  p.R = R;
  p.S = S;
  p.Hq = Hq;
  p.Hk = Hk;
  p.L = L;
  p.nsplit = nsplit;
  p.scale = scale;
  p.ws = reinterpret_cast<float*>(ws);
  p.counters = counters;
  p.err = err;
  p.cluster = 0;
  cudaError_t e;
  switch (hd) {
    case 128: e = attn_tc_enabled() ? launch_attn_tc(p, R / S, pdl, stream) : launch_attn<128>(p, pdl, stream); break;
    case 256: e = launch_attn<256>(p, pdl, stream); break;
    case 384: e = launch_attn<384>(p, pdl, stream); break;
    default: return HM_EARG;
  }
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

// ------------------------------------------------------------------ allocation-free variant
// Some callers cannot allocate device memory when they run this kernel: a host
// that drives decoding from a real-time audio thread (cudaMalloc/cudaFree may
// synchronise the device and stall for milliseconds), or an application that
// hands out all device memory from its own fixed arena and forbids the CUDA
// allocator.  For them hm_decode_attn_noalloc keeps its scratch -- the split
// partials and the merge tickets -- in this fixed array instead of taking a
// workspace.  Every GPU that loads the library holds the array until exit.
constexpr size_t kNoAllocPartialFloats = size_t(1) << 20;  // 4 MiB of split partials
constexpr int kNoAllocTickets = 4096;
static __device__ __align__(256) float hm_attn_scratch[kNoAllocPartialFloats + kNoAllocTickets];

namespace {
constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  The array's name
// in host code is only a stand-in, so the address is looked up once per device
// (on that device's first call) and cached.
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, hm_attn_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}
}  // namespace

extern "C" int hm_decode_attn_noalloc(const void* q, const void* kc, const void* vc, const int64_t* pos, void* o,
                                      int R, int S, int Hq, int Hk, int hd, int L, float scale, int nsplit, int* err,
                                      hm_stream_t stream) {
  if (!q || !kc || !vc || !pos || !o || R < 1 || S < 1 || R % S || Hk < 1 || Hq % Hk || Hq / Hk > kMaxG || L < 1 ||
      nsplit < 1 || nsplit > kMaxSplit)
    return HM_EARG;
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15u) return HM_EARG;
  if (hd != 128 && hd != 256 && hd != 384) return HM_EARG;
  if (nsplit > 1 && (hm_decode_attn_workspace_bytes(R, Hq, hd, nsplit) > kNoAllocPartialFloats * sizeof(float) ||
                     R * Hk > kNoAllocTickets))
    return HM_ENOSPACE;
  void* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess) return static_cast<int>(e);
  float* partials = reinterpret_cast<float*>(base);
  int* tickets = reinterpret_cast<int*>(partials + kNoAllocPartialFloats);
  if (nsplit > 1) {
    // the array keeps whatever the previous call left: start from zero tickets
    e = cudaMemsetAsync(tickets, 0, sizeof(int) * R * Hk, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  AttnParams p;
  p.q = reinterpret_cast<const __half*>(q);
  p.kc = reinterpret_cast<const __half*>(kc);
  p.vc = reinterpret_cast<const __half*>(vc);
  p.pos = pos;
  p.o = reinterpret_cast<__half*>(o);
  p.R = R;
  p.S = S;
  p.Hq = Hq;
  p.Hk = Hk;
  p.L = L;
  p.nsplit = nsplit;
  p.scale = scale;
  p.ws = partials;
  p.counters = tickets;
  p.err = err;
  p.cluster = 0;
  switch (hd) {
    case 128: e = launch_attn<128>(p, 0, stream); break;
    case 256: e = launch_attn<256>(p, 0, stream); break;
    default: e = launch_attn<384>(p, 0, stream); break;
  }
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
