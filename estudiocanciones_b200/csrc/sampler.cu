// Fused CFG + top-k + exponential-race sampler for one codebook (sm_100a).
//
// Replaces `_guided` + `_sample` (app/engine.py:291-305) — in the reference a
// chain of ~10 torch kernels per codebook (mix, /temp, topk, masked_fill,
// log_softmax, softmax, exponential_, div, argmax, cat).  The exponential
// noise is an input (drawn by torch's generator so the random stream matches
// the reference), everything else is one CTA per take:
//   l   = (CFG ? u + fp16(fp16(c - u) * cfg) : c) / temp          (fp16 mix, fp32 divide)
//   thr = k-th largest l  (radix select on order-preserving keys)
//   l'  = l >= thr ? l : -inf
//   p   = softmax(log_softmax(l'))                                  (fp32)
//   id  = argmax(p / noise)   (first index on ties, NaN counts as largest)
#include "hm_common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kPer = 9;  // values per thread: V <= 9216
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

__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// block-wide reductions with a fixed combination order (deterministic)
__device__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[l];
  r = warp_max(r);
  return r;
}
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[l];
  r = warp_sum(r);
  return r;
}

// (value, index) argmax: larger value wins, NaN beats numbers, ties -> smaller index
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  const bool na = isnan(a), nb = isnan(b);
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

__global__ void __launch_bounds__(kThreads) sampler_kernel(const __grid_constant__ SampParams P) {
  __shared__ int hist[256];
  __shared__ float red[kWarps];
  __shared__ float rv[kWarps];
  __shared__ int ri[kWarps];
  __shared__ uint32_t sel_s;
  __shared__ int kk_s;
  pdl_trigger();
  pdl_wait();
  const int n = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // parameters in registers (the block barriers below would force re-reads otherwise)
  const int V = P.V, Nt = P.N, topk = P.topk;
  const bool mix = P.B == 2 * Nt;
  const float cfg = P.cfg, temp = P.temp;
  const __half* const logits = P.logits;
  const int64_t ldl = P.ld_logits, ldn = P.ld_noise, out_ld = P.out_ld;
  const float* const noise = P.noise;
  int64_t* const outp = P.out;
  const int out_col = P.out_col;
  int* const err = P.err;
  float l[kPer];
  uint32_t key[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = tid + j * kThreads;
    float val = -INFINITY;
    if (v < V) {
      const __half c = logits[(int64_t)n * ldl + v];
      __half g = c;
      if (mix) {
        const __half u = logits[(int64_t)(n + Nt) * ldl + v];
        const __half d = __hsub(c, u);
        const __half e = __float2half_rn(__half2float(d) * cfg);
        g = __hadd(u, e);
      }
      val = __fdiv_rn(__half2float(g), temp);
    }
    l[j] = val;
    key[j] = f2key(val);
  }

  // ---- radix select of the topk-th largest key, 8 bits per pass from the top
  uint32_t prefix = 0, pmask = 0;
  int kk = topk;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int v = tid + j * kThreads;
      const bool in = v < V && (key[j] & pmask) == prefix;
      const uint32_t dig = (key[j] >> shift) & 255u;
      const uint32_t act = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t peers = __match_any_sync(act, dig);
        if ((__ffs(peers) - 1) == lane) atomicAdd(&hist[dig], __popc(peers));
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns digits [248 - 8l, 255 - 8l], scanned from the top
      int cnt[8];
      int tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cnt[i] = hist[255 - 8 * lane - i];
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
            sel_s = 255u - 8u * lane - i;
            kk_s = kk - cum;
            break;
          }
          cum += cnt[i];
        }
      }
      if (who == 0 && lane == 0) {  // fewer than topk values: keep everything
        sel_s = 0;
        kk_s = 1;
      }
    }
    __syncthreads();
    prefix |= sel_s << shift;
    pmask |= 255u << shift;
    kk = kk_s;
    __syncthreads();
  }
  const float thr = key2f(prefix);

  // ---- softmax(log_softmax(masked)) and the exponential race
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (!(l[j] >= thr)) l[j] = -INFINITY;
    mx = fmaxf(mx, l[j]);
  }
  mx = block_max(mx, red);
  float se = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) se += l[j] == -INFINITY ? 0.f : expf(l[j] - mx);
  se = block_sum(se, red);
  const float lz = logf(se);
  float mx2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    l[j] = l[j] == -INFINITY ? -INFINITY : (l[j] - mx) - lz;
    mx2 = fmaxf(mx2, l[j]);
  }
  mx2 = block_max(mx2, red);
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    l[j] = l[j] == -INFINITY ? 0.f : expf(l[j] - mx2);
    s2 += l[j];
  }
  s2 = block_sum(s2, red);
  float best = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int v = tid + j * kThreads;
    if (v < V) {
      const float r = __fdiv_rn(__fdiv_rn(l[j], s2), noise[(int64_t)n * ldn + v]);
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
    rv[warp] = best;
    ri[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = rv[lane];
    bi = ri[lane];
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
      if (bi < 0 || bi >= V) {
        report_error(err, HM_ERR_BADINDEX);
        bi = 0;
      }
      outp[(int64_t)n * out_ld + out_col] = bi;
      if (mix) outp[(int64_t)(n + Nt) * out_ld + out_col] = bi;
    }
  }
}

}  // namespace

extern "C" int hm_cfg_topk_sample(const void* logits, int64_t ld_logits, int B, int N, int V, const float* noise,
                                  int64_t ld_noise, float cfg, int topk, float temp, int64_t* out, int64_t out_ld,
                                  int out_col, int* err, int pdl, hm_stream_t stream) {
  if (!logits || !noise || !out || N < 1 || (B != N && B != 2 * N) || V < 1 || V > kThreads * kPer || topk < 1 ||
      topk > V)
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
  const cudaError_t e = hm_launch(sampler_kernel, dim3(N), dim3(kThreads), 0, stream, pdl, p);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
