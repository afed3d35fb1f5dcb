// Small per-row kernels of the HeartMuLa decode path (sm_100a).
//
// These back the reference's standalone entry points (`rms`, `_rope_cache`,
// `_silu_mul` in app/kernels.py, `Emb.__call__` and the frame's embedding sum
// in app/engine.py).  The fused decode path folds RMSNorm, RoPE and SiLU into
// the GEMV (gemv_i8.cu); what remains per frame here is the embedding sum that
// starts the backbone and the frame-commit bookkeeping at the end.
#include "hm_common.cuh"

namespace {

// ------------------------------------------------------------------ RMSNorm
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                                      __half* __restrict__ y, int D, float eps) {
  __shared__ float red[8];
  __shared__ float inv_s;
  const int r = blockIdx.x, tid = threadIdx.x;
  const __half* xr = x + (int64_t)r * D;
  float a = 0.f;
  for (int k = tid; k < D; k += 256) {
    const float v = __half2float(xr[k]);
    a += v * v;
  }
  a = warp_sum(a);
  if ((tid & 31) == 0) red[tid >> 5] = a;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    inv_s = 1.0f / sqrtf(s / static_cast<float>(D) + eps);
  }
  __syncthreads();
  const float inv = inv_s;
  for (int k = tid; k < D; k += 256)
    y[(int64_t)r * D + k] = hmul_rn(__float2half_rn(__half2float(xr[k]) * inv), w[k]);
}

// Same arithmetic on 8-element chunks (16-byte loads and stores): the prompt-prefill
// shape (thousands of rows of 3072) is pure HBM traffic, read once and written once.
__global__ void __launch_bounds__(128) rmsnorm8_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                                       __half* __restrict__ y, int D, float eps) {
  __shared__ float red[4];
  const int r = blockIdx.x, tid = threadIdx.x, nc = D / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)r * D);
  float a = 0.f;
  for (int c = tid; c < nc; c += 128) {
    const uint4 v = xr[c];
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
      a += f.x * f.x;
      a += f.y * f.y;
    }
  }
  a = warp_sum(a);
  if ((tid & 31) == 0) red[tid >> 5] = a;
  __syncthreads();
  const float inv = 1.0f / sqrtf((((red[0] + red[1]) + red[2]) + red[3]) / static_cast<float>(D) + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + (int64_t)r * D);
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  for (int c = tid; c < nc; c += 128) {
    const uint4 v = xr[c], g = w4[c];
    uint4 o;
    o.x = rms_h2(v.x, g.x, inv);
    o.y = rms_h2(v.y, g.y, inv);
    o.z = rms_h2(v.z, g.z, inv);
    o.w = rms_h2(v.w, g.w, inv);
    yr[c] = o;
  }
}

// ------------------------------------------------------------------ RMSNorm from sum-of-squares partials
// out[r, k] = fp16(fp16(x[r, k] * inv_r) * gamma[k]) with inv_r = 1/sqrt(sum_t ss[t, r] / dim + eps),
// the partials written by the producer of x (16 columns each).  Every CTA reduces the
// partials of all rows (a few KB, 16-byte loads) in the same order as the GEMV's fused
// RMSNorm prologue, then normalises its 1024-column slice: the same values, computed once
// per launch instead of once per GEMV CTA.
__global__ void __launch_bounds__(128) rms_apply_kernel(const __half* __restrict__ x, int64_t ldx,
                                                        const float* __restrict__ ss, int ss_tiles, int64_t ss_ld,
                                                        const __half* __restrict__ gamma, float eps, int dim,
                                                        __half* __restrict__ out, int64_t ldo, int R, int D) {
  constexpr int kMaxR = 32;
  __shared__ float part[4][kMaxR];
  __shared__ float inv_s[kMaxR];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nv = (R + 3) / 4;
  float a[kMaxR];
#pragma unroll
  for (int i = 0; i < kMaxR; ++i) a[i] = 0.f;
  for (int t = tid; t < ss_tiles; t += 128) {
    const float4* p4 = reinterpret_cast<const float4*>(ss + (int64_t)t * ss_ld);
#pragma unroll
    for (int j = 0; j < kMaxR / 4; ++j) {
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
  for (int i = 0; i < kMaxR; ++i)
    if (i < 4 * nv) a[i] = warp_sum(a[i]);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < kMaxR; ++i)
      if (i < R) part[warp][i] = a[i];
  }
  __syncthreads();
  if (tid < R) {
    const float tot = ((part[0][tid] + part[1][tid]) + part[2][tid]) + part[3][tid];
    inv_s[tid] = 1.0f / sqrtf(tot / static_cast<float>(dim) + eps);
  }
  __syncthreads();
  const int c = blockIdx.x * 128 + tid;  // 8-column chunk
  if (8 * c >= D) return;
  const uint4 gv = reinterpret_cast<const uint4*>(gamma)[c];
  for (int r = 0; r < R; ++r) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + (int64_t)r * ldx + 8 * c);
    const float inv = inv_s[r];
    uint4 o;
    o.x = rms_h2(v.x, gv.x, inv);
    o.y = rms_h2(v.y, gv.y, inv);
    o.z = rms_h2(v.z, gv.z, inv);
    o.w = rms_h2(v.w, gv.w, inv);
    *reinterpret_cast<uint4*>(out + (int64_t)r * ldo + 8 * c) = o;
  }
}

// ------------------------------------------------------------------ RoPE + KV-cache write
__global__ void rope_kv_kernel(const __half* __restrict__ qkv, const float* __restrict__ rope, int rope_rows,
                               const int64_t* __restrict__ pos, __half* __restrict__ q_out, __half* __restrict__ kc,
                               __half* __restrict__ vc, int S, int Hq, int Hk, int hd, int L, int* err) {
  const int r = blockIdx.x, h = blockIdx.y, i = threadIdx.x;  // pair (2i, 2i+1)
  if (2 * i >= hd) return;
  const int64_t p = pos[r];
  if (p < 0 || p >= L || p >= rope_rows) {
    if (i == 0) report_error(err, HM_ERR_BADINDEX);
    return;
  }
  const int b = r / S;
  const int W = (Hq + 2 * Hk) * hd;
  const float c = rope[(p * (hd / 2) + i) * 2], sn = rope[(p * (hd / 2) + i) * 2 + 1];
  if (h < Hq) {
    const __half* src = qkv + (int64_t)r * W + h * hd + 2 * i;
    const float x0 = __half2float(src[0]), x1 = __half2float(src[1]);
    __half* dst = q_out + (int64_t)r * Hq * hd + h * hd + 2 * i;
    dst[0] = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    dst[1] = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
  } else {
    const int kh = h - Hq;
    const __half* src = qkv + (int64_t)r * W + (Hq + kh) * hd + 2 * i;
    const float x0 = __half2float(src[0]), x1 = __half2float(src[1]);
    const int64_t dst = (((int64_t)b * Hk + kh) * L + p) * hd + 2 * i;
    kc[dst] = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    kc[dst + 1] = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
    const __half* vs = qkv + (int64_t)r * W + (Hq + Hk + kh) * hd + 2 * i;
    vc[dst] = vs[0];
    vc[dst + 1] = vs[1];
  }
}

// Same rotation, 8 head dims (4 pairs) per thread: one 16-byte qkv load, two 16-byte
// table loads, one 16-byte store (and the 16-byte V copy for a K head).  Threads of
// a row run over its heads' chunks in order, so every load and store is coalesced.
__device__ __forceinline__ uint32_t rot_h2(uint32_t xv, float c, float sn) {
  const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&xv));
  const __half lo = __float2half_rn(__fsub_rn(__fmul_rn(x.x, c), __fmul_rn(x.y, sn)));
  const __half hi = __float2half_rn(__fadd_rn(__fmul_rn(x.y, c), __fmul_rn(x.x, sn)));
  return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

__global__ void __launch_bounds__(256) rope_kv8_kernel(const __half* __restrict__ qkv, const float* __restrict__ rope,
                                                       int rope_rows, const int64_t* __restrict__ pos,
                                                       __half* __restrict__ q_out, __half* __restrict__ kc,
                                                       __half* __restrict__ vc, int R, int S, int Hq, int Hk, int hd,
                                                       int L, int* err) {
  const int cph = hd / 8, cpr = (Hq + Hk) * cph;
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (int64_t)R * cpr) return;
  const int r = static_cast<int>(idx / cpr), c = static_cast<int>(idx % cpr);
  const int h = c / cph, j = c % cph;
  const int64_t p = pos[r];
  if (p < 0 || p >= L || p >= rope_rows) {
    if (c == 0) report_error(err, HM_ERR_BADINDEX);
    return;
  }
  const int64_t W = (int64_t)(Hq + 2 * Hk) * hd;
  const float4* t4 = reinterpret_cast<const float4*>(rope + (p * (hd / 2) + 4 * j) * 2);
  const float4 t0 = t4[0], t1 = t4[1];  // (cos, sin) of pairs 4j .. 4j+3
  const uint4 xv = *reinterpret_cast<const uint4*>(qkv + (int64_t)r * W + (int64_t)h * hd + 8 * j);
  uint4 o;
  o.x = rot_h2(xv.x, t0.x, t0.y);
  o.y = rot_h2(xv.y, t0.z, t0.w);
  o.z = rot_h2(xv.z, t1.x, t1.y);
  o.w = rot_h2(xv.w, t1.z, t1.w);
  if (h < Hq) {
    *reinterpret_cast<uint4*>(q_out + (int64_t)r * Hq * hd + (int64_t)h * hd + 8 * j) = o;
  } else {
    const int kh = h - Hq, b = r / S;
    const int64_t dst = (((int64_t)b * Hk + kh) * L + p) * hd + 8 * j;
    *reinterpret_cast<uint4*>(kc + dst) = o;
    *reinterpret_cast<uint4*>(vc + dst) =
        *reinterpret_cast<const uint4*>(qkv + (int64_t)r * W + (int64_t)(h + Hk) * hd + 8 * j);
  }
}

// ------------------------------------------------------------------ SiLU * mul
__global__ void silu_mul_kernel(const __half* __restrict__ a, __half* __restrict__ y, int F) {
  const int r = blockIdx.x;
  const int c = blockIdx.y * 256 + threadIdx.x;
  if (c >= F) return;
  const float af = __half2float(a[(int64_t)r * 2 * F + c]);
  const __half s = __float2half_rn(__fdiv_rn(af, __fadd_rn(1.0f, expf(-af))));
  y[(int64_t)r * F + c] = hmul_rn(s, a[(int64_t)r * 2 * F + F + c]);
}

// ------------------------------------------------------------------ int8 embedding gather
__global__ void emb_gather_kernel(const int64_t* __restrict__ idx, const int8_t* __restrict__ tab,
                                  const __half* __restrict__ scale, int64_t rows, int D, __half* __restrict__ out,
                                  int* err) {
  const int i = blockIdx.x;
  const int64_t id = idx[i];
  if (id < 0 || id >= rows) {
    if (threadIdx.x == 0) report_error(err, HM_ERR_BADINDEX);
    for (int k = threadIdx.x; k < D; k += blockDim.x) out[(int64_t)i * D + k] = __float2half_rn(0.f);
    return;
  }
  const float s = __half2float(scale[id]);
  for (int k = threadIdx.x; k < D; k += blockDim.x)
    out[(int64_t)i * D + k] = __float2half_rn(static_cast<float>(tab[id * D + k]) * s);
}

// Sum of the n_cb codebook embeddings of each row (fp32 accumulation, one
// rounding) and per-16-column sums of squares of the fp16 result (the
// granularity every residual-stream producer writes for the fused RMSNorm).
__global__ void __launch_bounds__(256) emb_sum_kernel(const int64_t* __restrict__ tok, int64_t tok_ld, int ncb,
                                                      int64_t vocab, const int8_t* __restrict__ tab,
                                                      const __half* __restrict__ scale, int64_t rows, int D,
                                                      __half* __restrict__ x, float* __restrict__ ss, int64_t ss_ld,
                                                      int* err) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.y, tid = threadIdx.x;
  const int k = blockIdx.x * 256 + tid;
  float a = 0.f;
  if (k < D) {
    for (int c = 0; c < ncb; ++c) {
      const int64_t id = tok[(int64_t)r * tok_ld + c] + c * vocab;
      if (id < 0 || id >= rows) {
        report_error(err, HM_ERR_BADINDEX);
        continue;
      }
      a += __half2float(__float2half_rn(static_cast<float>(tab[id * D + k]) * __half2float(scale[id])));
    }
  }
  const __half v = __float2half_rn(a);
  if (k < D) x[(int64_t)r * D + k] = v;
  if (ss) {
    float q = k < D ? __half2float(v) * __half2float(v) : 0.f;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if ((tid & 15) == 0 && k < D) ss[(int64_t)(k / 16) * ss_ld + r] = q;
  }
}

// ------------------------------------------------------------------ frame commit
// End of one decode frame: tok_in <- tok_out (next frame's input), stream[f] <-
// tok_out[:n_keep], pos += 1 for every row, frame counter += 1.
__global__ void frame_commit_kernel(const int64_t* __restrict__ tok_out, int64_t* __restrict__ tok_in, int B, int ncb,
                                    int64_t* __restrict__ pos, int n_keep, int64_t* __restrict__ stream,
                                    int64_t* __restrict__ frame, int64_t max_frames, int64_t* __restrict__ ends,
                                    int64_t eos_id) {
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  const int64_t f = *frame;
  // EOS tracking (generate's scan, app/engine.py:432-437): the first stream frame >= 1 in
  // which any codebook id of take b is >= eos_id, kept in ends[b] (-1 until then)
  if (ends && f >= 1)
    for (int b = tid; b < n_keep; b += blockDim.x) {
      bool eos = false;
      for (int j = 0; j < ncb; ++j) eos |= tok_out[b * ncb + j] >= eos_id;
      if (eos && ends[b] < 0) ends[b] = f;
    }
  for (int i = tid; i < B * ncb; i += blockDim.x) {
    const int64_t v = tok_out[i];
    tok_in[i] = v;
    const int b = i / ncb;
    if (stream && b < n_keep && f >= 0 && f < max_frames) stream[f * n_keep * ncb + i] = v;
  }
  __syncthreads();
  if (tid < B) pos[tid] += 1;
  if (tid == 0) *frame = f + 1;
}

}  // namespace

extern "C" int hm_rmsnorm(const void* x, const void* w, void* y, int R, int D, float eps, hm_stream_t stream) {
  if (!x || !w || !y || R < 1 || D < 1) return HM_EARG;
  if (D % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                       reinterpret_cast<uintptr_t>(y)) & 15u) == 0)
    rmsnorm8_kernel<<<R, 128, 0, stream>>>(reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(w),
                                           reinterpret_cast<__half*>(y), D, eps);
  else
    rmsnorm_kernel<<<R, 256, 0, stream>>>(reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(w),
                                          reinterpret_cast<__half*>(y), D, eps);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_rms_apply(const void* x, int64_t ldx, const float* ss, int ss_tiles, int64_t ss_ld,
                            const void* gamma, float eps, int dim, void* out, int64_t ldo, int R, int D, int pdl,
                            hm_stream_t stream) {
  if (!x || !ss || !gamma || !out || R < 1 || R > 32 || D < 8 || D % 8 || ss_tiles < 1 || dim < 1) return HM_EARG;
  if ((ss_ld & 3) || ldx % 8 || ldo % 8 ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(gamma) |
        reinterpret_cast<uintptr_t>(ss)) & 15u))
    return HM_EARG;
  const cudaError_t e =
      hm_launch(rms_apply_kernel, dim3((D / 8 + 127) / 128), dim3(128), 0, stream, pdl,
                reinterpret_cast<const __half*>(x), ldx, ss, ss_tiles, ss_ld, reinterpret_cast<const __half*>(gamma),
                eps, dim, reinterpret_cast<__half*>(out), ldo, R, D);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_rope_kv_write(const void* qkv, const float* rope, int rope_rows, const int64_t* pos, void* q_out,
                                void* kc, void* vc, int R, int S, int Hq, int Hk, int hd, int L, int* err,
                                hm_stream_t stream) {
  if (!qkv || !rope || !pos || !q_out || !kc || !vc || R < 1 || S < 1 || hd < 2 || hd % 2 || hd > 2048 || Hq < 1 ||
      Hk < 1)
    return HM_EARG;
  const bool vec = hd % 8 == 0 && ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(rope) |
                                    reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(kc) |
                                    reinterpret_cast<uintptr_t>(vc)) & 15u) == 0;
  if (vec) {
    const int64_t n = (int64_t)R * (Hq + Hk) * (hd / 8);
    rope_kv8_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        reinterpret_cast<const __half*>(qkv), rope, rope_rows, pos, reinterpret_cast<__half*>(q_out),
        reinterpret_cast<__half*>(kc), reinterpret_cast<__half*>(vc), R, S, Hq, Hk, hd, L, err);
  } else {
    rope_kv_kernel<<<dim3(R, Hq + Hk), hd / 2, 0, stream>>>(
        reinterpret_cast<const __half*>(qkv), rope, rope_rows, pos, reinterpret_cast<__half*>(q_out),
        reinterpret_cast<__half*>(kc), reinterpret_cast<__half*>(vc), S, Hq, Hk, hd, L, err);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_silu_mul(const void* a, void* y, int R, int F, hm_stream_t stream) {
  if (!a || !y || R < 1 || F < 1) return HM_EARG;
  silu_mul_kernel<<<dim3(R, (F + 255) / 256), 256, 0, stream>>>(reinterpret_cast<const __half*>(a),
                                                               reinterpret_cast<__half*>(y), F);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_emb_gather_i8(const int64_t* idx, int n, const int8_t* tab, const void* scale, int64_t rows, int D,
                                void* out, int* err, hm_stream_t stream) {
  if (!idx || !tab || !scale || !out || n < 1 || D < 1) return HM_EARG;
  emb_gather_kernel<<<n, 256, 0, stream>>>(idx, tab, reinterpret_cast<const __half*>(scale), rows, D,
                                           reinterpret_cast<__half*>(out), err);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_emb_sum_i8(const int64_t* tok, int64_t tok_ld, int R, int ncb, int64_t vocab, const int8_t* tab,
                             const void* scale, int64_t rows, int D, void* x_out, float* ss_out, int64_t ss_ld,
                             int* err, int pdl, hm_stream_t stream) {
  if (!tok || !tab || !scale || !x_out || R < 1 || ncb < 1 || D < 1 || (ss_out && D % 16)) return HM_EARG;
  const cudaError_t e = hm_launch(emb_sum_kernel, dim3((D + 255) / 256, R), dim3(256), 0, stream, pdl, tok, tok_ld,
                                  ncb, vocab, tab, reinterpret_cast<const __half*>(scale), rows, D,
                                  reinterpret_cast<__half*>(x_out), ss_out, ss_ld, err);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

extern "C" int hm_frame_commit(const int64_t* tok_out, int64_t* tok_in, int B, int ncb, int64_t* pos, int n_keep,
                               int64_t* stream_out, int64_t* frame, int64_t max_frames, int64_t* ends, int64_t eos_id,
                               int pdl, hm_stream_t stream) {
  if (!tok_out || !tok_in || !pos || !frame || B < 1 || B > 1024 || ncb < 1 || n_keep < 0 || n_keep > B) return HM_EARG;
  const cudaError_t e = hm_launch(frame_commit_kernel, dim3(1), dim3(256), 0, stream, pdl, tok_out, tok_in, B, ncb,
                                  pos, n_keep, stream_out, frame, max_frames, ends, eos_id);
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
