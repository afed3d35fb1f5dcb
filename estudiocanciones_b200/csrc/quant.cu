// Symmetric per-row int8 quantisation of a weight or embedding matrix on the GPU: the
// checkpoint converter's q8_rows (app/convert_final.py:17-21).
//
//   s[r]    = max(max_k |x[r,k]|, 1e-8) / 127                      (fp32)
//   q[r, k] = int8(clamp(round_half_even(x[r,k] / s[r]), -127, 127))
//
// s is stored as bf16 (round to nearest even), the format the converter saves.  The
// maximum is exact in any order, and the two divisions are IEEE round-to-nearest, as
// torch's are, so q and s are bit-identical to the converter's (NaN inputs aside).
//
// HBM-bound byte work: one CTA per row (grid-stride over rows), the row read once to
// find its maximum and again (from L2, which holds the rows in flight) to quantise;
// 16-byte loads and 4-byte stores where the row layout allows.
#include "hm_common.cuh"

#include <cuda_bf16.h>

namespace {

constexpr int kQThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// four consecutive elements as floats (p 4-element aligned when vec)
template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
  } else {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    const T* h = reinterpret_cast<const T*>(&a);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = to_f32<T>(h[i]);
  }
}

__device__ __forceinline__ int8_t q8_of(float x, float s) {
  const float v = fminf(fmaxf(rintf(__fdiv_rn(x, s)), -127.f), 127.f);
  return static_cast<int8_t>(static_cast<int>(v));
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kQThreads) q8_rows_kernel(const T* __restrict__ x, int64_t N, int64_t K, int64_t ldx,
                                                            int8_t* __restrict__ q, int64_t ldq,
                                                            __nv_bfloat16* __restrict__ s) {
  __shared__ float wmax[kQThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t r = blockIdx.x; r < N; r += gridDim.x) {
    const T* xr = x + r * ldx;
    int8_t* qr = q + r * ldq;
    float m = 0.f;
    if (VEC) {
      for (int64_t k = 4 * (int64_t)tid; k < K; k += 4 * kQThreads) {
        float v[4];
        load4<T>(xr + k, v);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
      }
    } else {
      for (int64_t k = tid; k < K; k += kQThreads) m = fmaxf(m, fabsf(to_f32<T>(xr[k])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[warp] = m;
    __syncthreads();
    float amax = wmax[0];
#pragma unroll
    for (int w = 1; w < kQThreads / 32; ++w) amax = fmaxf(amax, wmax[w]);
    const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.f);
    if (VEC) {
      for (int64_t k = 4 * (int64_t)tid; k < K; k += 4 * kQThreads) {
        float v[4];
        load4<T>(xr + k, v);
        char4 c;
        c.x = q8_of(v[0], sc);
        c.y = q8_of(v[1], sc);
        c.z = q8_of(v[2], sc);
        c.w = q8_of(v[3], sc);
        *reinterpret_cast<char4*>(qr + k) = c;
      }
    } else {
      for (int64_t k = tid; k < K; k += kQThreads) qr[k] = q8_of(to_f32<T>(xr[k]), sc);
    }
    if (tid == 0) s[r] = __float2bfloat16_rn(sc);
    __syncthreads();  // wmax is rewritten by the next row
  }
}

template <typename T>
cudaError_t launch_q8(const void* x, int64_t N, int64_t K, int64_t ldx, int8_t* q, int64_t ldq, void* s,
                      cudaStream_t st) {
  int nsm = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = static_cast<int64_t>(nsm > 0 ? nsm : 148) * 8;  // 8 CTAs of 256 threads per SM
  const dim3 grid(static_cast<unsigned>(N < cap ? N : cap));
  const uintptr_t align = sizeof(T) * 4;
  const bool vec = K % 4 == 0 && ldx % 4 == 0 && ldq % 4 == 0 && (reinterpret_cast<uintptr_t>(x) % align) == 0 &&
                   (reinterpret_cast<uintptr_t>(q) % 4) == 0;
  const T* xt = static_cast<const T*>(x);
  __nv_bfloat16* sb = static_cast<__nv_bfloat16*>(s);
  if (vec)
    q8_rows_kernel<T, true><<<grid, kQThreads, 0, st>>>(xt, N, K, ldx, q, ldq, sb);
  else
    q8_rows_kernel<T, false><<<grid, kQThreads, 0, st>>>(xt, N, K, ldx, q, ldq, sb);
  return cudaGetLastError();
}

}  // namespace

extern "C" int hm_q8_rows(const void* x, int dtype, int64_t N, int64_t K, int64_t ldx, int8_t* q, int64_t ldq,
                          void* s, hm_stream_t stream) {
  if (!x || !q || !s || N < 1 || K < 1 || ldx < K || ldq < K) return HM_EARG;
  cudaError_t e;
  switch (dtype) {
    case HM_DT_F32: e = launch_q8<float>(x, N, K, ldx, q, ldq, s, stream); break;
    case HM_DT_BF16: e = launch_q8<__nv_bfloat16>(x, N, K, ldx, q, ldq, s, stream); break;
    case HM_DT_F16: e = launch_q8<__half>(x, N, K, ldx, q, ldq, s, stream); break;
    default: return HM_EARG;
  }
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}

// ------------------------------------------------------------------ int8 -> fp16 (exact, unscaled)
// The prompt prefill multiplies by the weights as fp16 values on the tensor cores; every
// int8 value is exact in fp16 and the per-row scale is applied to the fp32 sums in the
// GEMM's epilogue, so converting once per layer and prompt (instead of in every CTA of
// the GEMM that reads the tile) changes no result.  HBM-bound: 1 byte read and 2 written
// per element, 16-byte loads and 2 x 16-byte stores, grid-stride.
namespace {
__global__ void __launch_bounds__(256) dequant_i8_kernel(const uint4* __restrict__ w, uint4* __restrict__ out,
                                                         int64_t n16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 q = __ldcs(w + i);
    uint4 h0, h1;
    i8x4_to_h2x2(q.x, h0.x, h0.y);
    i8x4_to_h2x2(q.y, h0.z, h0.w);
    i8x4_to_h2x2(q.z, h1.x, h1.y);
    i8x4_to_h2x2(q.w, h1.z, h1.w);
    out[2 * i] = h0;
    out[2 * i + 1] = h1;
  }
}
}  // namespace

extern "C" int hm_dequant_i8_f16(const int8_t* w, void* out, int64_t n, hm_stream_t stream) {
  if (!w || !out || n < 16 || n % 16 || ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15u))
    return HM_EARG;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n16 = n / 16;
  const int64_t want = (n16 + 255) / 256;
  const int grid = static_cast<int>(want < 8LL * sms ? want : 8LL * sms);
  dequant_i8_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const uint4*>(w), reinterpret_cast<uint4*>(out), n16);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
