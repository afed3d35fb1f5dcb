// Causal GQA prefill attention over the static KV cache (sm_100a tensor cores).
//
// Replaces the prompt branch of the reference's attention in Block.__call__
// (app/engine.py:123-153): for a prompt of P positions the reference expands K/V
// over the query heads (repeat_interleave) and calls SDPA with is_causal.  Here
// K/V are read once per KV head from the cache the RoPE/KV-write step filled,
// and shared by the G = Hq/Hk query heads of that KV head (no copy).
//
//   o[b*P + p, h*hd + d] = sum_{j <= p} softmax_j(q_p . k_j * scale) v_j[d]
//
// One CTA = (64 query positions, one KV head, one batch row); 4 warps per query
// head, 16 positions each.  K/V tiles of 64 positions x 128 dims arrive by 2-D
// TMA (128B swizzle) through a 2-stage ring; QK^T and PV are mma.sync m16n8k16
// (fp16 in, fp32 accumulate), the online softmax stays in registers and the
// probabilities are rounded to fp16 for PV (FA2 scheme).  Heavy (late) query
// tiles are scheduled first.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "hm_common.cuh"

namespace {

constexpr int kPos = 64;    // positions per K/V tile and per query tile
constexpr int kNst = 2;
constexpr int kBox = kPos * 128;  // bytes of one 64-position x 64-dim fp16 box
constexpr int kMaxGq = 4;

struct PaSmem {
  uint8_t k[kNst][2][kBox];
  uint8_t v[kNst][2][kBox];
  uint64_t bar[kNst];
  int abort_flag;
};

struct PaParams {
  const __half* q;
  __half* o;
  int B, P, Hq, Hk, L;
  float scale;
  int* err;
};

__device__ __forceinline__ uint32_t swz(const uint8_t* box, int row, int chunk) {
  return smem_u32(box + row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(G * 128, 1) prefill_attn_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                  const __grid_constant__ CUtensorMap vmap,
                                                                  const __grid_constant__ PaParams Pp) {
  constexpr int HD = 128;
  extern __shared__ uint8_t smem_raw[];
  PaSmem& sm = *reinterpret_cast<PaSmem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int P = Pp.P, Hq = Pp.Hq, Hk = Pp.Hk, L = Pp.L;
  const int nqt = (P + kPos - 1) / kPos;
  const int qt = nqt - 1 - (int)blockIdx.x;  // late (long) query tiles first
  const int kh = blockIdx.y, b = blockIdx.z;
  const int head = kh * G + warp / 4;
  const int qrow0 = qt * kPos + 16 * (warp & 3);  // first query position of this warp
  const float scale = Pp.scale;
  int* const err = Pp.err;
  volatile int* abort_s = &sm.abort_flag;

  if (tid == 0) {
    sm.abort_flag = 0;
    for (int i = 0; i < kNst; ++i) mbar_init(&sm.bar[i], 1);
    fence_barrier_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  __syncthreads();

  const int ntile = qt + 1;  // causal: K/V tiles 0 .. qt
  const int row0 = (b * Hk + kh) * L;
  auto issue = [&](int tt) {
    const int st = tt % kNst;
    const int y = row0 + tt * kPos;
    mbar_arrive_expect_tx(&sm.bar[st], 4 * kBox);
    tma_load_2d_plain(sm.k[st][0], &kmap, 0, y, &sm.bar[st]);
    tma_load_2d_plain(sm.k[st][1], &kmap, 64, y, &sm.bar[st]);
    tma_load_2d_plain(sm.v[st][0], &vmap, 0, y, &sm.bar[st]);
    tma_load_2d_plain(sm.v[st][1], &vmap, 64, y, &sm.bar[st]);
  };
  if (tid == 0)
    for (int tt = 0; tt < kNst && tt < ntile; ++tt) issue(tt);

  // q rows qrow0+g and qrow0+g+8 of this warp's head, as A fragments for 8 k-steps
  uint32_t qa[8][4];
  {
    const int64_t ld = (int64_t)Hq * HD;
    const int pa = qrow0 + g, pb = qrow0 + g + 8;
    const __half* qa_p = Pp.q + ((int64_t)b * P + pa) * ld + (int64_t)head * HD;
    const __half* qb_p = Pp.q + ((int64_t)b * P + pb) * ld + (int64_t)head * HD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = pa < P ? *reinterpret_cast<const uint32_t*>(qa_p + 16 * ks + 2 * t) : 0u;
      qa[ks][1] = pb < P ? *reinterpret_cast<const uint32_t*>(qb_p + 16 * ks + 2 * t) : 0u;
      qa[ks][2] = pa < P ? *reinterpret_cast<const uint32_t*>(qa_p + 16 * ks + 8 + 2 * t) : 0u;
      qa[ks][3] = pb < P ? *reinterpret_cast<const uint32_t*>(qb_p + 16 * ks + 8 + 2 * t) : 0u;
    }
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int mi = lane >> 3, ri = lane & 7;

  for (int tt = 0; tt < ntile; ++tt) {
    const int st = tt % kNst;
    mbar_wait_ab(&sm.bar[st], (tt / kNst) & 1, err, abort_s);  // on timeout: carry on, error flagged
    if (tt * kPos + kPos > P) {
      // last tile reaches past the prompt: its masked probabilities are 0, but
      // 0 * (non-finite cache contents) would not be, so zero those V rows
      const int nv = P - tt * kPos;
      for (int i = tid; i < 2 * (kPos - nv) * 8; i += G * 128) {
        const int box = i / ((kPos - nv) * 8), rem = i % ((kPos - nv) * 8);
        *reinterpret_cast<uint4*>(sm.v[st][box] + (nv + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
      }
      __syncthreads();
    }
    // ---- S = Q K^T: 16 query rows x 64 keys (8 n-tiles of 8 keys)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int kp = np * 16 + (mi >= 2 ? 8 : 0) + ri;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int c = 2 * ks + (mi & 1);
        uint32_t b00, b01, b10, b11;
        ldsm_x4(b00, b01, b10, b11, swz(sm.k[st][c >> 3], kp, c & 7));
        mma_16816(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b00, b01);
        mma_16816(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b10, b11);
      }
    }
    // ---- causal mask, scale, online softmax (rows g: e = 0,1; row g+8: e = 2,3)
    const int key0 = tt * kPos;
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + 8 * n + 2 * t + (e & 1);
        const int qp = qrow0 + g + (e >= 2 ? 8 : 0);
        const float v = key <= qp ? s[n][e] * scale : -INFINITY;
        s[n][e] = v;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 1));
      tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 2));
      const float m_new = fmaxf(m_run[h], tmax[h]);
      alpha[h] = (m_new == -INFINITY || m_run[h] == -INFINITY) ? (m_new == -INFINITY ? 1.f : 0.f)
                                                                : expf(m_run[h] - m_new);
      m_run[h] = m_new;
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = (s[n][e] == -INFINITY) ? 0.f : expf(s[n][e] - m_run[h]);
        s[n][e] = p;
        psum[h] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * alpha[h] + psum[h];  // quad-partial sums
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      acc[i][0] *= alpha[0];
      acc[i][1] *= alpha[0];
      acc[i][2] *= alpha[1];
      acc[i][3] *= alpha[1];
    }
    // ---- acc += fp16(P) V over 4 k-steps of 16 keys
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa0 = pack_h2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t pa1 = pack_h2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t pa2 = pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t pa3 = pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      const int vp = kk * 16 + (mi & 1) * 8 + ri;
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        const int c = 2 * nd + (mi >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(v0, v1, v2, v3, swz(sm.v[st][c >> 3], vp, c & 7));
        mma_16816(acc[2 * nd], pa0, pa1, pa2, pa3, v0, v1);
        mma_16816(acc[2 * nd + 1], pa0, pa1, pa2, pa3, v2, v3);
      }
    }
    __syncthreads();  // every warp is done with stage st
    if (tid == 0 && tt + kNst < ntile) issue(tt + kNst);
  }

  // ---- normalise and store rows g and g+8
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  const int64_t ld = (int64_t)Hq * HD;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int p = qrow0 + g + 8 * h;
    if (p >= P) continue;
    const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
    __half* op = Pp.o + ((int64_t)b * P + p) * ld + (int64_t)head * HD;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<uint32_t*>(op + 8 * i + 2 * t) = pack_h2(acc[i][2 * h] * inv, acc[i][2 * h + 1] * inv);
  }
}

// [rows, 128] fp16 view of a K or V cache, 64-dim x 64-position boxes, 128B swizzle
bool kv_map(const void* base, int64_t rows, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::pair<int64_t, CUtensorMap>> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(base);
    if (it != cache.end() && it->second.first == rows) {
      *out = it->second.second;
      return true;
    }
  }
  auto enc = hm_encode_fn();
  if (!enc) return false;
  CUtensorMap m;
  cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kPos)};
  cuuint32_t es[2] = {1, 1};
  if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache[base] = {rows, m};
  *out = m;
  return true;
}

template <int G>
cudaError_t launch_pa(const CUtensorMap& km, const CUtensorMap& vm, const PaParams& p, dim3 grid, hm_stream_t st) {
  const size_t smem = sizeof(PaSmem) + 1024;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return hm_launch(prefill_attn_kernel<G>, grid, dim3(128 * G), smem, st, false, km, vm, p);
}

}  // namespace

extern "C" int hm_prefill_attn(const void* q, const void* kc, const void* vc, void* o, int B, int P, int Hq, int Hk,
                               int hd, int L, float scale, int* err, hm_stream_t stream) {
  if (!q || !kc || !vc || !o || B < 1 || P < 1 || Hk < 1 || Hq < Hk || Hq % Hk != 0 || hd != 128 || P > L)
    return HM_EARG;
  if (Hq / Hk > kMaxGq) return HM_EARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(kc) |
       reinterpret_cast<uintptr_t>(vc)) & 15u)
    return HM_EARG;
  const int64_t rows = (int64_t)B * Hk * L;
  CUtensorMap km, vm;
  if (!kv_map(kc, rows, &km) || !kv_map(vc, rows, &vm)) return HM_EARG;
  PaParams p;
  p.q = reinterpret_cast<const __half*>(q);
  p.o = reinterpret_cast<__half*>(o);
  p.B = B;
  p.P = P;
  p.Hq = Hq;
  p.Hk = Hk;
  p.L = L;
  p.scale = scale;
  p.err = err;
  const dim3 grid((P + kPos - 1) / kPos, Hk, B);
  cudaError_t e;
  switch (Hq / Hk) {
    case 1: e = launch_pa<1>(km, vm, p, grid, stream); break;
    case 2: e = launch_pa<2>(km, vm, p, grid, stream); break;
    case 3: e = launch_pa<3>(km, vm, p, grid, stream); break;
    default: e = launch_pa<4>(km, vm, p, grid, stream); break;
  }
  return e == cudaSuccess ? HM_OK : static_cast<int>(e);
}
