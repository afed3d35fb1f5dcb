/*
 * heartmula_b200.h — C ABI of the B200 (sm_100a) HeartMuLa decode-path library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as `hm_stream_t`), launches on that stream, never allocates and
 * never synchronises, so all of them can be captured into a CUDA graph.
 * Each returns 0 on success, a cudaError_t value (> 0) when the launch failed,
 * or HM_EARG (< 0) when an argument is out of the supported range.
 *
 * Device-side faults are not used for error reporting: kernels that can meet a
 * bad index or a wait that never ends OR a bit (HM_ERR_*) into the caller's
 * `err` word (a device int, may be NULL) and skip the access / return.
 *
 * Activations are fp16 (IEEE half stored as uint16), weights int8 row-major
 * [N, K] with one fp16 scale per row, matching the reference checkpoint after
 * its loader (app/engine.py:235-242 casts the bf16 scales to fp16).
 */
#ifndef HEARTMULA_B200_H
#define HEARTMULA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hm_stream_t; /* == cudaStream_t */

/* host return codes */
#define HM_OK 0
#define HM_EARG (-1)
#define HM_ENOSPACE (-2) /* the request needs more than a fixed space holds (hm_decode_attn_noalloc's scratch
                            array, a stage sequence's shared-memory activation region) */

/* element types of hm_q8_rows' input */
#define HM_DT_F32 0
#define HM_DT_BF16 1
#define HM_DT_F16 2

/* device error-word bits */
#define HM_ERR_TIMEOUT 1   /* a bounded wait gave up */
#define HM_ERR_BADINDEX 2  /* token id / position outside its table; access skipped */

/* ------------------------------------------------------------------ int8 GEMV
 * y[m, n] = fp16( sum_k x[m,k] * w[n,k] * s[n] ) (+ res[m, n] in fp16),  M <= 32, K % 16 == 0.
 * Replaces int8_mm / _gemv8 (app/kernels.py:20-54; M <= 16 branch, extended to 32).
 * `ws`/`counters`: split-K scratch, sized by hm_gemv_workspace_bytes /
 * hm_gemv_counters; counters must be zero before the first call and are left
 * zero by every call.  kspan = 0 picks the split automatically; kspan > 0 splits K into
 * k-ranges of kspan columns reduced through `ws` (the last CTA of a tile sums them);
 * kspan = -s (s = 2, 4 or 8) splits K over the s CTAs of a thread-block cluster, reduced
 * in distributed shared memory (no scratch; bit-identical to kspan = K / s). */
int hm_gemv_i8(const void* x, int64_t ldx, const int8_t* w, const void* s, const void* res, int64_t ldres, void* y,
               int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes, int* counters, int n_counters, int* err,
               int kspan, int pdl, hm_stream_t stream);

/* Where the GEMV input rows come from (fused prologue). */
#define HM_SRC_F16 0 /* x row as is */
#define HM_SRC_RMS 1 /* RMSNorm of the x row: fp16(fp16(x*inv)*gamma), inv from ss partials (app/kernels.py:58-67) */
#define HM_SRC_EMB 2 /* int8 embedding row fp16(q8[id]*s8[id]) with id = tok[...] + tok_off (app/engine.py:95-98) */

typedef struct {
  int mode;
  int row_mul, row_add;         /* source row of output row m: m*row_mul + row_add */
  const void* x;                /* F16/RMS: fp16 rows */
  int64_t ldx;
  const float* ss;              /* RMS: sum-of-squares partials ss[t*ss_ld + row], t < ss_tiles */
  int ss_tiles;
  int64_t ss_ld;
  const void* gamma;            /* RMS: fp16 [K] */
  float eps;
  int dim;                      /* RMS: row width D (divisor of the mean) */
  const int8_t* etab;           /* EMB: int8 table [erows, K] */
  const void* escale;           /* EMB: fp16 [erows] */
  int64_t erows;
  const int64_t* tok;           /* EMB: id = tok[row*tok_ld + tok_col] + tok_off */
  int64_t tok_ld;
  int tok_col;
  int64_t tok_off;
} hm_row_src;

#define HM_EPI_STORE 0   /* y = fp16(acc*s) (+res); optional per-16-column sum of squares */
#define HM_EPI_ROPE_KV 1 /* fused qkv: RoPE q -> q_out, RoPE k / copy v -> cache slot pos (app/kernels.py:79-107) */
#define HM_EPI_SILU 2    /* fused w1|w3: y[m,j] = fp16(silu(a)) * b (app/kernels.py:172-180) */

typedef struct {
  const int8_t* w;
  const void* s;
  int N, K, M;
  hm_row_src src[2];
  int interleave;               /* 1: row m takes src[m & 1] with local row m >> 1 */
  int epi;
  void* y;                      /* STORE/SILU output */
  int64_t ldy;
  const void* res;              /* STORE: optional residual (may alias y) */
  int64_t ldres;
  float* ss_out;                /* STORE: optional ss partials ss_out[t*ss_out_ld + m], t = 16-column tile */
  int64_t ss_out_ld;
  const float* rope;            /* ROPE_KV: fp32 [rope_rows, hd/2, 2] */
  int rope_rows;
  const int64_t* pos;           /* ROPE_KV: absolute position of each row */
  int S, Hq, Hk, hd, L;         /* ROPE_KV: rows per batch entry, heads, head dim, cache length */
  void* q_out;                  /* ROPE_KV: fp16 [M, Hq*hd] */
  void* kc;                     /* ROPE_KV: fp16 [B, Hk, L, hd] */
  void* vc;
  void* ws;                     /* split-K scratch */
  size_t ws_bytes;
  int* counters;
  int n_counters;
  int* err;
  int kspan;                    /* 0 = automatic, > 0 k-range width, -2/-4/-8 cluster split */
  int pdl;                      /* launch with programmatic dependent launch */
  int l2_keep;                  /* weights read again soon (decoder passes): L2 evict-last instead of evict-first */
} hm_gemv_desc;

/* The fused GEMV: prologue rows from `src`, epilogue per `epi`.  The per-layer
 * decode path of Stack.decode (app/engine.py:180-211) is five of these plus
 * hm_decode_attn. */
int hm_gemv_i8_fused(const hm_gemv_desc* d, hm_stream_t stream);

/* Scratch needed by a GEMV of this shape (kspan = 0: the automatic choice). */
size_t hm_gemv_workspace_bytes(int M, int N, int K, int epi, int kspan);
int hm_gemv_counters(int N, int epi);
/* The split actually used for a shape (for reporting). */
int hm_gemv_pick_kspan(int M, int N, int K, int epi, int kspan);

/* ------------------------------------------------------------------ small kernels */
/* rms(x, w, eps) (app/kernels.py:58-74). x, y fp16 [R, D]; w fp16 [D]. */
int hm_rmsnorm(const void* x, const void* w, void* y, int R, int D, float eps, hm_stream_t stream);

/* RMSNorm from the sum-of-squares partials a residual producer wrote (ss[t*ss_ld + r],
 * 16 columns each): out = fp16(fp16(x * 1/sqrt(sum/dim + eps)) * gamma), R <= 32 rows,
 * D % 8 == 0, 16-byte aligned.  Same values as the GEMV's fused RMSNorm prologue
 * (app/kernels.py:58-67 rounding), computed once per launch. */
int hm_rms_apply(const void* x, int64_t ldx, const float* ss, int ss_tiles, int64_t ss_ld, const void* gamma,
                 float eps, int dim, void* out, int64_t ldo, int R, int D, int pdl, hm_stream_t stream);

/* _rope_cache (app/kernels.py:79-107): qkv [R, (Hq+2Hk)*hd] -> q_out [R, Hq*hd],
 * kc/vc [B, Hk, L, hd] written at pos[r] for batch r / S. */
int hm_rope_kv_write(const void* qkv, const float* rope, int rope_rows, const int64_t* pos, void* q_out, void* kc,
                     void* vc, int R, int S, int Hq, int Hk, int hd, int L, int* err, hm_stream_t stream);

/* _silu_mul (app/kernels.py:172-180): a [R, 2F] -> y [R, F]. */
int hm_silu_mul(const void* a, void* y, int R, int F, hm_stream_t stream);

/* Emb.__call__ int8 branch (app/engine.py:95-98): out[i] = fp16(q8[idx[i]] * s8[idx[i]]). */
int hm_emb_gather_i8(const int64_t* idx, int n, const int8_t* tab, const void* scale, int64_t rows, int D, void* out,
                     int* err, hm_stream_t stream);

/* Backbone input of a frame (app/engine.py:348): x[r] = fp16(sum_c emb(tok[r,c] + c*vocab)),
 * plus optional ss partials per 16 columns for the next fused RMSNorm. */
int hm_emb_sum_i8(const int64_t* tok, int64_t tok_ld, int R, int ncb, int64_t vocab, const int8_t* tab,
                  const void* scale, int64_t rows, int D, void* x_out, float* ss_out, int64_t ss_ld, int* err, int pdl,
                  hm_stream_t stream);

/* End of one decode frame (the bookkeeping of generate's loop, app/engine.py:419-437,
 * kept on the device): tok_in <- tok_out, stream[frame] <- tok_out[:n_keep],
 * pos[b] += 1, frame += 1.  tok_* are int64 [B, ncb]; stream int64 [max_frames, n_keep, ncb].
 * EOS tracking (ends may be NULL): ends[b] (int64 [n_keep], -1 = none yet) <- frame, the
 * first stream frame >= 1 in which any id of take b is >= eos_id (the reference's EOS scan
 * of out[1:], AUDIO_EOS = 8193), so the host reads n_keep integers instead of scanning. */
/* ------------------------------------------------------------------ checkpoint conversion
 * q8_rows of the converter (app/convert_final.py:17-21) on the GPU: x [N, K] (row pitch
 * ldx elements, type HM_DT_*) -> q int8 [N, K] (row pitch ldq), s bf16 [N] with
 * s[r] = max(max|x[r]|, 1e-8) / 127 and q = clamp(round_half_even(x / s), -127, 127);
 * bit-identical to the converter's torch arithmetic. */
int hm_q8_rows(const void* x, int dtype, int64_t N, int64_t K, int64_t ldx, int8_t* q, int64_t ldq, void* s,
               hm_stream_t stream);

int hm_frame_commit(const int64_t* tok_out, int64_t* tok_in, int B, int ncb, int64_t* pos, int n_keep,
                    int64_t* stream_out, int64_t* frame, int64_t max_frames, int64_t* ends, int64_t eos_id, int pdl,
                    hm_stream_t stream);

/* ------------------------------------------------------------------ decode attention
 * _attn + _attn_combine (app/kernels.py:112-167): row r of batch r/S attends
 * cache positions [0, pos[r]] with GQA (no KV copy); split over `nsplit`
 * position ranges, the last CTA of each (row, kv head) merges the partials.
 * q, o fp16 [R, Hq*hd]; kc, vc fp16 [B, Hk, L, hd]; hd in {128, 256, 384} (HM_EARG otherwise);
 * hd 128 runs the tensor-core kernel, 256 and 384 the CUDA-core one.
 * With pdl = 1 the launch reads `pos` and the cache slots before pos[r] before it
 * waits for the preceding launch (to overlap that launch's tail): the preceding
 * launch may write q and the slot at pos[r] (the fused qkv GEMV does), not those. */
int hm_decode_attn(const void* q, const void* kc, const void* vc, const int64_t* pos, void* o, int R, int S, int Hq,
                   int Hk, int hd, int L, float scale, int nsplit, void* ws, size_t ws_bytes, int* counters,
                   int n_counters, int* err, int pdl, hm_stream_t stream);
size_t hm_decode_attn_workspace_bytes(int R, int Hq, int hd, int nsplit);

/* Decode attention that allocates nothing (no counterpart in the reference, which
 * always takes its scratch from the torch allocator).  For callers that cannot
 * allocate device memory while they decode -- a real-time audio thread, where
 * cudaMalloc may synchronise the device and stall, or an application that serves
 * every buffer from its own fixed arena.  Same arguments as hm_decode_attn without
 * the workspace, and the same results within fp16 rounding: it always runs the
 * CUDA-core split kernel (also for hd 128, where hm_decode_attn uses the tensor-core
 * kernel, so the two differ in fp32 summation order).  The split partials and merge
 * tickets live in a fixed array inside the library (4 MiB of partials:
 * R*Hq*nsplit*(hd+2) floats <= 1048576, and R*Hk <= 4096 tickets); larger requests
 * return HM_ENOSPACE.  Every GPU that loads the library holds the array until the
 * process exits.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and keeps it for the process, so make that first call before
 * any stream capture; the kept address does not survive cudaDeviceReset (or any other
 * reset of the device's primary context): after one, do not call this entry point again
 * in that process.  All calls share the one array: calls that overlap on the GPU (other
 * streams, other threads) race on it. */
int hm_decode_attn_noalloc(const void* q, const void* kc, const void* vc, const int64_t* pos, void* o, int R, int S,
                           int Hq, int Hk, int hd, int L, float scale, int nsplit, int* err, hm_stream_t stream);

/* ------------------------------------------------------------------ sampler
 * _guided + _sample (app/engine.py:291-305) for one codebook: optional CFG mix
 * (rows [0,N) conditional, [N,2N) unconditional, fp16 arithmetic), /temp,
 * top-k mask, softmax(log_softmax), argmax(p / noise).  The id is written to
 * out[b*out_ld + out_col] for b = n and, with CFG, b = n + N. */
int hm_cfg_topk_sample(const void* logits, int64_t ld_logits, int B, int N, int V, const float* noise,
                       int64_t ld_noise, float cfg, int topk, float temp, int64_t* out, int64_t out_ld, int out_col,
                       int* err, int pdl, hm_stream_t stream);

/* ------------------------------------------------------------------ prompt prefill
 * Tensor-core GEMM with int8 weights for many rows (tcgen05 MMA, fp32 accumulators in TMEM):
 *   epi HM_EPI_STORE: c[m, n] = fp16( sum_k a[m,k] * w[n,k] * s[n] ) (+ res[m, n] in fp16)
 *   epi HM_EPI_SILU : w = [w1; w3] (N = 2F rows), c[m, f] = fp16( fp16(silu(a1)) * a3 ), f < F,
 *                     a1/a3 the rounded w1/w3 outputs (res must be NULL)
 * K % 64 == 0, output columns % 16 == 0, lda/ldc/ldr % 8 == 0, 16-byte aligned pointers; c may equal res.
 * Replaces the M > 16 branch of int8_mm (app/kernels.py:46-49: dequantise, fp16 GEMM) used by
 * the prompt pass of Block.__call__ (app/engine.py:123-153). */
int hm_gemm_i8w(const void* a, int64_t lda, const int8_t* w, const void* s, const void* res, int64_t ldr, void* c,
                int64_t ldc, int M, int N, int K, int epi, int* err, hm_stream_t stream);

/* The same GEMM with the weights already in fp16 (w [N, K] fp16 holding the exact int8
 * values, from hm_dequant_i8_f16; s, epilogues and limits as hm_gemm_i8w, results
 * identical): the tensor cores read the weight tiles as TMA writes them, with no
 * per-tile conversion.  The prompt pass converts each layer's weights once per prompt. */
int hm_gemm_f16w(const void* a, int64_t lda, const void* w, const void* s, const void* res, int64_t ldr, void* c,
                 int64_t ldc, int M, int N, int K, int epi, int* err, hm_stream_t stream);

/* out[i] = (fp16) w[i] for n int8 values (exact; no scale): the weights of hm_gemm_f16w.
 * n % 16 == 0, 16-byte aligned pointers.  The dequantisation of int8_mm's M > 16 branch
 * (app/kernels.py:46-49) without the scale, which hm_gemm_f16w applies to the sums. */
int hm_dequant_i8_f16(const int8_t* w, void* out, int64_t n, hm_stream_t stream);

/* Causal GQA attention of a whole prompt over the cache positions [0, P) that the
 * RoPE/KV-write step filled: q, o [B*P, Hq*hd] fp16 (row b*P + p), kc/vc [B, Hk, L, hd].
 * hd == 128, Hq/Hk <= 4.  Replaces the prompt branch of Block.__call__'s attention
 * (repeat_interleave + SDPA is_causal, app/engine.py:123-153). */
int hm_prefill_attn(const void* q, const void* kc, const void* vc, void* o, int B, int P, int Hq, int Hk, int hd,
                    int L, float scale, int* err, hm_stream_t stream);

/* ------------------------------------------------------------------ HeartCodec detokenize
 * The codec turns the [8, T] token streams into audio (app/codec_lite.py:63-75 ->
 * HeartCodec.detokenize, app/heartcodec/modeling_heartcodec.py:57-204): a flow-matching
 * Euler solve over a LlamaTransformer estimator (models/flow_matching.py:72-210,
 * models/transformer.py) and the ScalarModel waveform decoder (models/sq_codec.py:506-510).
 *
 * hm_conv1d_gemm: every GEMM-shaped codec layer (nn.Linear, Conv1d, causal ConvTranspose1d,
 * the PostProcessor's repeat + conv) as one implicit-GEMM convolution on the tensor cores:
 *   acc[b, t, n] = sum_{j < taps} sum_{c < cin} x[b, t + off0 + j*dil, c] * w[j, n, c],
 * x rows outside [0, tin) reading as zero; then v = act((acc + bias[n]) * scale) and
 *   HM_CEPI_STORE : y = v                              (fp16, or fp32 with y_f32)
 *   HM_CEPI_GATED : y = res + gate[b*gate_ld + n] * v   (res, y fp32; y may equal res)
 *   HM_CEPI_RES   : y = v + res                        (res, y fp16; ResidualUnit's skip)
 *   HM_CEPI_SILU  : w rows in blocks of 256 (128 gate rows, the same 128 features' up rows),
 *                   y[f] = silu(v_gate) * v_up, f < N/2 (LlamaMLP; N % 256 == 0)
 *   HM_CEPI_ROPE  : columns n < rope_cols rotated in pairs (n even, n + 1) by rope[t][(n % hd)/2]
 *                   = (cos, sin) (LlamaAttention's apply_rope_vec on q and k)
 * Rows: input item b, row t at x + b*x_bstride + t*x_ld; output row b*T + t at y + row*y_ld
 * (res the same with res_ld).  cin % 64 == 0, npad % 64 == 0 (w holds npad >= N rows per
 * tap, the extra rows unused), x_ld/x_bstride % 8 == 0, 16-byte aligned x, w, y.
 * bn: single-SM tile width 64/128/256; -128 / -256: tiles of 256 rows on SM pairs (a cluster of two
 * CTAs, tcgen05 cta_group::2, same results bit for bit); 0 = automatic. */
#define HM_ACT_NONE 0
#define HM_ACT_PRELU 1
#define HM_ACT_SILU 2
#define HM_CEPI_STORE 0
#define HM_CEPI_GATED 1
#define HM_CEPI_RES 2
#define HM_CEPI_SILU 3
#define HM_CEPI_ROPE 4
typedef struct {
  const void* x;
  int64_t x_ld, x_bstride;
  const void* w;
  const float* bias;
  void* y;
  int64_t y_ld;
  const void* res;
  int64_t res_ld;
  const float* gate;
  int64_t gate_ld;
  const float* rope;
  int* err;
  int B, T, tin, cin, N, npad, taps, off0, dil;
  float scale, prelu;
  int act, epi, y_f32, rope_cols, hd, bn;
} hm_conv_desc;
int hm_conv1d_gemm(const hm_conv_desc* d, hm_stream_t stream);

/* Non-causal multi-head attention of the codec's estimator (LlamaAttention with SDPA,
 * models/transformer.py:129-145): q, k, v fp16 [B*T, ld] with head h at columns h*hd
 * (views into one fused q|k|v buffer), o fp16 [B*T, ldo]; hd 64 or 128. */
int hm_codec_attn(const void* q, const void* k, const void* v, void* o, int B, int T, int H, int hd, int64_t ld,
                  int64_t ldo, float scale, int* err, hm_stream_t stream);

/* out[b*T + t] = fp16( norm(x[b*T + t]) * (1 + scale[b*mod_ld + :]) + shift[b*mod_ld + :] ):
 * layer_norm 0: RMSNorm with weight w (models/transformer.py:9-18), 1: LayerNorm without
 * affine (nn.LayerNorm(elementwise_affine=False), :283-284); the ada-norm modulation of
 * LlamaTransformerBlock (:185-201) and of the estimator's output norms (:323-331, 345-350). */
int hm_codec_norm_mod(const float* x, int64_t ldx, const float* w, const float* shift, const float* scale,
                      int64_t mod_ld, void* out, int64_t ldo, int B, int T, int D, float eps, int layer_norm,
                      hm_stream_t stream);

/* Residual-VQ code lookup and project_out (models/flow_matching.py:100-104):
 * out[t] = fp16( proj_w (sum_q codebooks[q][codes[q*ld_codes + t]]) + proj_b ), codes clamped
 * to [0, K) (app/codec_lite.py:72); codebooks fp32 [nq][K][cd], proj_w fp32 [dim][cd]. */
int hm_codec_vq_embed(const int64_t* codes, int64_t ld_codes, int nq, int Tc, const float* codebooks, int K, int cd,
                      const float* proj_w, const float* proj_b, void* out, int64_t ldo, int dim, hm_stream_t stream);

/* dst row rep*t + i = src row t (fp16; nearest upsampling along time, flow_matching.py:108-110). */
int hm_codec_upsample_rows(const void* src, int64_t lds, int rows, int cols, int rep, void* dst, int64_t ldd,
                           hm_stream_t stream);

/* One Euler step of solve_euler (models/flow_matching.py:161-210) on the fp32 latents x [T, C]:
 * v NULL: x = noise; else x += dt * (u + g (c - u)) (nb == 2: v rows [0,T) unconditional,
 * [T,2T) conditional) or x += dt * v (nb == 1); then rows < L_in = (1 - (1 - 1e-6) t_next)
 * noise + t_next inc (final: = inc), and unless final, fp16(x) goes to columns [0, C) of
 * the nb estimator-input items (item b row t at xin + b*xin_bstride + t*ldx); the first call
 * (v NULL) also writes fp16(inc) rows < L_in, zeros after, to their columns [C, 2C). */
int hm_codec_euler(const float* v, int nb, float* x, const float* noise, const float* inc, int T, int C, int L_in,
                   float dt, float g, float t_next, int final, void* xin, int64_t ldx, int64_t xin_bstride,
                   hm_stream_t stream);

/* Latents [T, nband*Cb] fp32 -> decoder input [nband, T, Cb] fp16, round(9x)/9
 * (modeling_heartcodec.py:185-193 band split, sq_codec.py:384-393 round_func9). */
int hm_codec_band_quant(const float* x, int T, int Cb, int nband, void* out, hm_stream_t stream);

/* From the embedded timesteps E [S, D] (fp32): act = fp16(silu(E)), shift = tab[0] + E,
 * scale = tab[1] + E (AdaLayerNormSingleFlow's SiLU input and the output-norm modulation,
 * models/transformer.py:323-331, 438-443). */
int hm_codec_temb_post(const float* E, int S, int D, const float* tab, void* act, float* shift, float* scale,
                       hm_stream_t stream);

/* Window assembly of detokenize (modeling_heartcodec.py:185-204): out[c][start + i] = cur[c][i],
 * blended over i < ovlp as out (1 - w_i) + cur w_i with w = linspace(0, 1, ovlp) in fp64. */
int hm_codec_overlap_add(const float* cur, int64_t cur_ld, float* out, int64_t out_ld, int C, int64_t start, int64_t n,
                         int64_t ovlp, hm_stream_t stream);

/* ------------------------------------------------------------------ info */
int hm_device_sm_count(int device);
/* Form of the TMA requests a launch would use (no counterpart in the reference, whose Triton
 * kernels load with plain pointer arithmetic): 1 = one 3-D / 4-D box per 8 KB GEMV weight stage
 * (K % 128 == 0) or per 16 KB K / V tile of the tensor-core decode attention, 0 = several 2-D
 * boxes (HM_GEMV_BOX=0 / HM_ATTN_BOX=0 in the environment, or a shape the 3-D map cannot
 * describe), HM_EARG for bad arguments.  Both forms fill shared memory identically. */
int hm_gemv_box_form(const int8_t* w, int N, int K, int epi);
int hm_decode_attn_box_form(const void* cache, int64_t rows);
/* sizeof / offsetof of the descriptor structs, for bindings to verify their layout:
 * 0 sizeof(hm_row_src), 1 sizeof(hm_gemv_desc), 2 offsetof(hm_gemv_desc, src),
 * 3 offsetof(hm_gemv_desc, ws), 4 offsetof(hm_gemv_desc, pdl), 5 offsetof(hm_gemv_desc, l2_keep),
 * 6 sizeof(hm_conv_desc), 7 offsetof(hm_conv_desc, B), 8 offsetof(hm_conv_desc, scale),
 * 9 offsetof(hm_conv_desc, bn). */
size_t hm_abi_layout(int which);
const char* hm_version(void);

#ifdef __cplusplus
}
#endif

#endif /* HEARTMULA_B200_H */
