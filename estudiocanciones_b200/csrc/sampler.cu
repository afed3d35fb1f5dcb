// Fused CFG + top-k + exponential-race sampler for one codebook (sm_100a).
//
// Replaces `_guided` + `_sample` (app/engine.py:291-305) — in the reference a
// chain of ~10 torch kernels per codebook (mix, /temp, topk, masked_fill,
// log_softmax, softmax, exponential_, div, argmax, cat).  The exponential
// noise is an input (drawn by torch's generator so the random stream matches
// the reference), everything else is one thread-block cluster per take:
//   l   = (CFG ? u + fp16(fp16(c - u) * cfg) : c) / temp          (fp16 mix, fp32 divide)
//   thr = k-th largest l  (radix select on order-preserving fp16 keys of the mix)
//   l'  = l >= thr ? l : -inf
//   p   = softmax(log_softmax(l'))                                  (fp32)
//   id  = argmax(p / noise)   (first index on ties, NaN counts as largest)
//
// The vocabulary row is split over the 8 CTAs of a cluster (~1k values each, 4-5 per
// thread).  The selection and reductions combine through distributed shared memory:
// each CTA publishes its digit histogram (and its largest key) for a radix pass, its
// partial softmax sums, and pushes its argmax candidate to CTA 0; every CTA reads the
// eight published values in rank order after a cluster barrier, so all of them select
// the same threshold and see the same sums (deterministic).  Five cluster barriers
// per take instead of the per-value work of a whole row on one SM.
#include "hm_common.cuh"

namespace {

constexpr int kCl = 8;          // CTAs per take (cluster size; ld_dsmem_u32_x8 reads eight ranks)
constexpr int kThreads = 256;
constexpr int kPer = 5;         // values per thread: V <= kCl * kThreads * kPer = 10240
constexpr int kWarps = kThreads / 32;

struct SampParams {
  const __half* logits;
  int64_t ld_logits;
  int B, N, V;
  const float* noise;
  int64_t ld_noise;
  float cfg, temp;
  int topk;
  int64_t* out;
  int64_t out_ld;
  int out_col;
  int* err;
};

// Order-preserving 16-bit keys of fp16 values (NaN with the sign bit clear sorts
// above +inf, as in torch.topk).  l = fp32(g) / temp is non-decreasing in g, so
// the k-th largest l is the quotient of the k-th largest g: the selection runs on
// the 16-bit fp16 keys (two 8-bit radix passes instead of four on fp32 keys).
__device__ __forceinline__ uint32_t h2key(__half h) {
  const uint32_t u = __half_as_ushort(h);
  return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u);
}
__device__ __forceinline__ __half key2h(uint32_t k) {
  return __ushort_as_half(static_cast<unsigned short>((k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu)));
}

// block-wide sum with a fixed combination order (deterministic)
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = l < kWarps ? red[l] : 0.f;
  r = warp_sum(r);
  return r;
}

// (value, index) argmax: larger value wins, NaN beats numbers, ties -> smaller index
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  const bool na = isnan(a), nb = isnan(b);
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

struct SampShared {
  int hist[2][8][256];     // per radix pass: 8 copies (lane & 7) keep same-digit lanes apart
  int pub_hist[2][256];    // this CTA's digit counts per pass, read by the cluster
  int glob[256];           // the cluster's counts of the current pass
  uint32_t pub_maxkey;     // this CTA's largest key, read by the cluster
  float pub_sum[2];        // this CTA's partial softmax sums, read by the cluster
  float cand_v[kCl];       // argmax candidates pushed to CTA 0
  int cand_i[kCl];
  float red[kWarps];
  float rv[kWarps];
  int ri[kWarps];
  uint32_t sel_s;
  int kk_s;
};

// Select the digit holding the kk-th largest key from the cluster's histogram sh.glob
// (warp 0; lane l owns digits 255-8l .. 248-8l, scanned from the top).
__device__ void select_digit(SampShared& sh, int kk) {
  const int lane = threadIdx.x & 31;
  int cnt[8];
  int tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    cnt[i] = sh.glob[255 - 8 * lane - i];
    tot += cnt[i];
  }
  int incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const int before = incl - tot;
  const bool here = before < kk && kk <= incl;
  const uint32_t who = __ballot_sync(0xffffffffu, here);
  if (here) {
    int cum = before;
    for (int i = 0; i < 8; ++i) {
      if (cum + cnt[i] >= kk) {
        sh.sel_s = 255u - 8u * lane - i;
        sh.kk_s = kk - cum;
        break;
      }
      cum += cnt[i];
    }
  }
  if (who == 0 && lane == 0) {  // fewer than topk values: keep everything
    sh.sel_s = 0;
    sh.kk_s = 1;
  }
}

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kThreads) sampler_kernel(const __grid_constant__ SampParams P) {
  __shared__ SampShared sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = static_cast<int>(cluster_ctarank());
  const int n = blockIdx.x / kCl;
  // parameters in registers (the block barriers below would force re-reads otherwise)
  const int V = P.V, Nt = P.N, topk = P.topk;
  const bool mix = P.B == 2 * Nt;
  const float cfg = P.cfg, temp = P.temp;
  const int64_t ldl = P.ld_logits, ldn = P.ld_noise;
  const int chunk = (V + kCl - 1) / kCl;
  const int v0 = rank * chunk, vend = min(V, v0 + chunk);  // this CTA's part of the row
  pdl_trigger();
  for (int i = tid; i < 2 * 8 * 256; i += kThreads) (&sh.hist[0][0][0])[i] = 0;
  if (tid == 0) sh.pub_maxkey = 0;
  // the noise comes from a full (non-programmatic) dependency: read it before the wait
  float nz[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = v0 + tid + j * kThreads;
    nz[j] = v < vend ? P.noise[(int64_t)n * ldn + v] : 1.f;
  }
  pdl_wait();
  // every load of the two rows first (predicated, all in flight together), then the mix
  // (plain loads: the rows are rewritten by the head GEMV before every sampler, so they
  // must not come through the non-coherent read-only path)
  const unsigned short* const crow = reinterpret_cast<const unsigned short*>(P.logits + (int64_t)n * ldl);
  const unsigned short* const urow =
      reinterpret_cast<const unsigned short*>(P.logits + (int64_t)(n + (mix ? Nt : 0)) * ldl);
  unsigned short cb[kPer], ub[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = v0 + tid + j * kThreads;
    cb[j] = v < vend ? crow[v] : 0;
    ub[j] = v < vend && mix ? urow[v] : 0;
  }
  __half gv[kPer];
  uint32_t key[kPer];
  uint32_t kmax = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = v0 + tid + j * kThreads;
    __half g = __ushort_as_half(cb[j]);
    if (mix) {
      const __half c = g, u = __ushort_as_half(ub[j]);
      const __half d = __hsub(c, u);
      const __half e = __float2half_rn(__half2float(d) * cfg);
      g = __hadd(u, e);
    }
    if (v >= vend) g = __float2half_rn(0.f);
    gv[j] = g;
    key[j] = h2key(g);
    if (v < vend) kmax = max(kmax, key[j]);
  }
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  __syncthreads();  // histograms and pub_maxkey zeroed
  if (lane == 0) atomicMax(&sh.pub_maxkey, kmax);

  // ---- radix select of the topk-th largest fp16 key over the cluster: high byte, then low byte
  uint32_t sel_key = 0, maxkey = 0;
  int kk = topk;
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    int* const h = &sh.hist[pass][lane & 7][0];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int v = v0 + tid + j * kThreads;
      if (v < vend && (pass == 0 || (key[j] >> 8) == sel_key))
        atomicAdd(&h[pass == 0 ? (key[j] >> 8) : (key[j] & 255u)], 1);
    }
    __syncthreads();
    {  // this CTA's counts (256 threads = 256 digits)
      int c = 0;
#pragma unroll
      for (int cp = 0; cp < 8; ++cp) c += sh.hist[pass][cp][tid];
      sh.pub_hist[pass][tid] = c;
    }
    cluster_sync_all();  // every CTA's counts (and largest key) published
    {
      uint32_t c8[kCl];
      ld_dsmem_u32_x8(&sh.pub_hist[pass][tid], c8);
      int c = 0;
#pragma unroll
      for (int r = 0; r < kCl; ++r) c += static_cast<int>(c8[r]);
      sh.glob[tid] = c;
    }
    if (pass == 0) {
      uint32_t k8[kCl];
      ld_dsmem_u32_x8(&sh.pub_maxkey, k8);
#pragma unroll
      for (int r = 0; r < kCl; ++r) maxkey = max(maxkey, k8[r]);
    }
    __syncthreads();
    if (warp == 0) select_digit(sh, kk);
    __syncthreads();
    sel_key = (sel_key << 8) | sh.sel_s;
    kk = sh.kk_s;
  }
  // Keep l >= k-th largest l.  For fp16 g and any temp in [1e-20, 1e20] the fp32
  // quotients of distinct g stay distinct (their relative gap, >= 2^-11, is far
  // above fp32 rounding, and they neither overflow nor underflow), so the test is
  // the fp16 comparison g >= g_k; outside that range the quotients are compared.
  const __half thr_h = key2h(sel_key);
  const float thr_g = __half2float(thr_h);
  const bool direct = temp >= 1e-20f && temp <= 1e20f;
  const float thr_l = __fdiv_rn(thr_g, temp);

  // ---- softmax(log_softmax(masked)): only kept values divide and exponentiate
  // the largest kept value is the quotient of the largest key (always kept)
  const float mx = __fdiv_rn(__half2float(key2h(maxkey)), temp);
  float l[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = v0 + tid + j * kThreads;
    const float gf = __half2float(gv[j]);
    const bool kept = v < vend && (direct ? gf >= thr_g : __fdiv_rn(gf, temp) >= thr_l);
    l[j] = -INFINITY;
    if (kept) l[j] = __fdiv_rn(gf, temp);
  }
  float se = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (l[j] != -INFINITY) se += expf(l[j] - mx);
  se = block_sum(se, sh.red);
  if (tid == 0) sh.pub_sum[0] = se;
  cluster_sync_all();
  {
    uint32_t s8[kCl];
    ld_dsmem_u32_x8(&sh.pub_sum[0], s8);
    se = 0.f;
#pragma unroll
    for (int r = 0; r < kCl; ++r) se += __uint_as_float(s8[r]);  // rank order: the same in every CTA
  }
  const float lz = logf(se);
  // max of the log-softmax is (mx - mx) - lz = -lz exactly: no reduction needed
  const float mx2 = -lz;
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (l[j] != -INFINITY) {
      l[j] = expf(((l[j] - mx) - lz) - mx2);
      s2 += l[j];
    } else {
      l[j] = 0.f;
    }
  }
  s2 = block_sum(s2, sh.red);
  if (tid == 0) sh.pub_sum[1] = s2;
  cluster_sync_all();
  {
    uint32_t s8[kCl];
    ld_dsmem_u32_x8(&sh.pub_sum[1], s8);
    s2 = 0.f;
#pragma unroll
    for (int r = 0; r < kCl; ++r) s2 += __uint_as_float(s8[r]);
  }
  // argmax(p / noise): a dropped value has p = 0, so 0 / noise is 0, or NaN when the
  // noise is 0 or NaN (NaN wins the argmax, as in torch)
  float best = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = v0 + tid + j * kThreads;
    if (v < vend) {
      float r;
      if (l[j] != 0.f) r = __fdiv_rn(__fdiv_rn(l[j], s2), nz[j]);
      else r = (nz[j] == 0.f || nz[j] != nz[j]) ? __int_as_float(0x7fffffff) : 0.f;
      if (better(r, v, best, bi)) {
        best = r;
        bi = v;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sh.rv[warp] = best;
    sh.ri[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kWarps ? sh.rv[lane] : -INFINITY;
    bi = lane < kWarps ? sh.ri[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, best, bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {  // this CTA's candidate into CTA 0's slot `rank`
      st_dsmem_f32(dsmem_addr(&sh.cand_v[rank], 0), best);
      st_dsmem_f32(dsmem_addr(&sh.cand_i[rank], 0), __int_as_float(bi));
    }
  }
  cluster_sync_all();  // after this only CTA 0 reads, its own shared memory
  if (rank == 0 && tid == 0) {
    best = sh.cand_v[0];
    bi = sh.cand_i[0];
    for (int r = 1; r < kCl; ++r)
      if (better(sh.cand_v[r], sh.cand_i[r], best, bi)) {
        best = sh.cand_v[r];
        bi = sh.cand_i[r];
      }
    if (bi < 0 || bi >= V) {
      report_error(P.err, HM_ERR_BADINDEX);
      bi = 0;
    }
    P.out[(int64_t)n * P.out_ld + P.out_col] = bi;
    if (mix) P.out[(int64_t)(n + Nt) * P.out_ld + P.out_col] = bi;
  }
}

}  // namespace

extern "C" int hm_cfg_topk_sample(const void* logits, int64_t ld_logits, int B, int N, int V, const float* noise,
                                  int64_t ld_noise, float cfg, int topk, float temp, int64_t* out, int64_t out_ld,
                                  int out_col, int* err, int pdl, hm_stream_t stream) {
  if (!logits || !noise || !out || N < 1 || (B != N && B != 2 * N) || V < 1 || V > kCl * kThreads * kPer ||
      topk < 1 || topk > V)
    return HM_EARG;
  SampParams p;
  p.logits = reinterpret_cast<const __half*>(logits);
  p.ld_logits = ld_logits;
  p.B = B;
  p.N = N;
  p.V = V;
  p.noise = noise;
  p.ld_noise = ld_noise;
  p.cfg = cfg;
  p.temp = temp;
  p.topk = topk;
  p.out = out;
  p.out_ld = out_ld;
  p.out_col = out_col;
  p.err = err;
  const cudaError_t e = hm_launch(sampler_kernel, dim3(N * kCl), dim3(kThreads), 0, stream, pdl, p);  // a cluster per take
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
