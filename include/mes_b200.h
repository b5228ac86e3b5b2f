/*
 * mes_b200 - C ABI of the B200 (sm_100a) kernels behind the embedding server's
 * GPU-worker forward pass.
 *
 * Conventions
 *   - Every pointer is a CUDA device pointer unless stated otherwise; tensors are dense
 *     row-major.  Element types are given per argument: bf16 = __nv_bfloat16,
 *     f16 = __half, i32 / i64 = int32_t / int64_t, f32 = float.
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued on it and the call
 *     returns without synchronising.  Nothing here allocates device memory: scratch
 *     comes from the caller.
 *   - The return value is a mes_status (0 = success).  Argument errors are detected on
 *     the host before anything is launched.  Device-side wait limits record a code that
 *     mes_take_device_error() returns.
 *   - Alignment: activation, weight, scale/zero-point and output arrays start on 16-byte
 *     boundaries (the kernels move them with TMA or as 16-byte vectors); index arrays
 *     (i64 ids, positions, row indices) on 8 bytes; the f32 residual R of
 *     mes_awq_gemm_residual on 4 and a GEMM bias on 2.  A pointer that does not returns
 *     MES_ERR_ALIGN (the repack and dequantisation helpers need element alignment only).
 *
 * Each entry point names the reference interface (woodx9/minimal-embedding-server, path
 * within that project, file:line) whose computation it replaces.
 */
#ifndef MES_B200_H_
#define MES_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mes_status {
  MES_OK = 0,
  MES_ERR_INVALID = 1,     /* bad size, null pointer or unsupported shape          */
  MES_ERR_ALIGN = 2,       /* pointer or pitch violates the stated alignment       */
  MES_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed                    */
  MES_ERR_TIMEOUT = 4,     /* a device wait ran past its limit (see device error)  */
  MES_ERR_UNSUPPORTED = 5  /* no sm_100a device / feature unavailable              */
} mes_status;

/* Library version (major*10000 + minor*100 + patch). */
int mes_version(void);

/* Human-readable text for a status code (static storage). */
const char* mes_status_string(int status);

/* Returns and clears the first device-side error code recorded by any kernel of this
 * library on the current device (0 if none).  Synchronises the current device. */
int mes_take_device_error(int* code);

/* Self-test of the bounded device wait that every pipeline role of this library uses: one
 * GPU thread waits on an mbarrier phase, with a limit of `limit_ns` (1 .. 1e8 ns).  With
 * `arrive` == 0 nothing completes the phase, so the wait runs out, records MES_ERR_TIMEOUT
 * (returned by the next mes_take_device_error) and the kernel returns normally - the
 * context stays usable; with `arrive` != 0 the thread arrives first and nothing is
 * recorded.  No counterpart in the reference, which has no device waits. */
int mes_wait_probe(int64_t limit_ns, int arrive, void* stream);

/* Leaves `sms` SMs (0..64) free of the persistent kernels (AWQ GEMM, attention) so that
 * another kernel running concurrently - an NCCL all-reduce overlapped on its own stream -
 * delays none of their CTAs.  Process-wide; 0 (the default) uses every SM.  No counterpart
 * in the reference, whose collectives do not overlap its GEMMs. */
int mes_set_sm_reserve(int sms);

/* ---------------------------------------------------------------------------------
 * Embedding gather.  out[t, :] = table[ids[t], :].
 * Replaces VocabParallelEmbedding.forward (layers/embed_head.py:43-52); the table is
 * replicated per rank, so no all-reduce is needed at tp>1.
 * ids: i64 [T] (each in [0, vocab)); table: bf16 [vocab, H]; out: bf16 [T, H]; H % 8 == 0.
 * Out-of-range ids produce a zero row and record MES_ERR_INVALID as device error.
 * ------------------------------------------------------------------------------- */
int mes_embedding(const int64_t* ids, int64_t T, const void* table, int64_t vocab,
                  int64_t H, void* out, void* stream);

/* Same gather widened exactly to f32 [T, H]: the start of the model's fp32 residual stream
 * (the reference keeps the residual in bf16: models/qwen3.py:131-133). */
int mes_embedding_f32(const int64_t* ids, int64_t T, const void* table, int64_t vocab,
                      int64_t H, float* out, void* stream);

/* ---------------------------------------------------------------------------------
 * RMSNorm.  y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w), statistics in fp32.
 * Replaces RMSNorm.rms_forward (layers/layernorm.py:18-27).
 * x, y: bf16 [rows, H] (y may alias x); w: bf16 [H]; H % 256 == 0, H <= 8192.
 * ------------------------------------------------------------------------------- */
int mes_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t H, float eps,
                void* stream);

/* RMSNorm of an f32 input (the fp32 residual stream) to bf16 y; same arithmetic. */
int mes_rmsnorm_f32in(const float* x, const void* w, void* y, int64_t rows, int64_t H,
                      float eps, void* stream);

/* ---------------------------------------------------------------------------------
 * Fused residual add + RMSNorm.  s = x + residual (fp32); residual_out = bf16(s);
 * y = bf16(bf16(s * rsqrt(mean(s^2) + eps)) * w).
 * Replaces RMSNorm.add_rms_forward (layers/layernorm.py:30-41).
 * x, residual: bf16 [rows, H]; y, residual_out: bf16 [rows, H].  y may alias x and
 * residual_out may alias residual (in-place update of the residual stream).
 * ------------------------------------------------------------------------------- */
int mes_add_rmsnorm(const void* x, const void* residual, const void* w, void* y,
                    void* residual_out, int64_t rows, int64_t H, float eps, void* stream);

/* Fused add + RMSNorm with a f32 residual stream: s = x + residual (x bf16 [rows, H],
 * residual f32 [rows, H] updated in place to s), y = bf16 RMSNorm(s) as above.  Used after
 * the tensor-parallel all-reduce of the o_proj / down_proj partial sums. */
int mes_add_rmsnorm_f32res(const void* x, float* residual, const void* w, void* y,
                           int64_t rows, int64_t H, float eps, void* stream);

/* ---------------------------------------------------------------------------------
 * Fused per-head q/k RMSNorm + NeoX RoPE, in place on the packed QKV projection output.
 * Replaces the q_norm/k_norm calls of Qwen3Attention.forward (models/qwen3.py:82-88) and
 * RotaryEmbedding.forward (layers/rotary_embedding.py:39-55; Qwen2: models/qwen2.py:85).
 * qkv: bf16 rows of pitch `ld` elements holding Hq q heads then Hkv k heads of D each
 *      (the packed [T, (Hq + 2*Hkv) * D] projection output; its v heads are untouched).
 *      Hq or Hkv may be 0 to rotate a q-only or k-only tensor.
 * positions: i64 [T]; cos_sin: bf16 or f32 (cos_sin_f32 != 0) [max_pos, D] = cat(cos, sin);
 * q_w, k_w: bf16 [D] (ignored when apply_norm == 0); D == 128.
 * ------------------------------------------------------------------------------- */
int mes_qknorm_rope(void* qkv, int64_t ld, const int64_t* positions, const void* cos_sin,
                    int cos_sin_f32, int64_t max_pos, const void* q_w, const void* k_w,
                    int64_t T, int Hq, int Hkv, int D, float eps, int apply_norm,
                    void* stream);

/* ---------------------------------------------------------------------------------
 * SiLU-and-mul.  y[r, i] = bf16(silu(x[r, i]) * x[r, I + i]) in fp32.
 * Replaces SiluAndMul.forward (layers/activation.py:12-14).
 * x: bf16 [rows, 2I]; y: bf16 [rows, I]; I % 8 == 0.
 * ------------------------------------------------------------------------------- */
int mes_silu_mul(const void* x, void* y, int64_t rows, int64_t I, void* stream);

/* ---------------------------------------------------------------------------------
 * Sequence boundaries and attention work list for a packed varlen batch, computed on
 * the device (no host synchronisation).  A new sequence starts at token i when
 * positions[i] != positions[i-1] + 1 - the rule of layers/attention/flashattention.py:26-34,
 * which the reference evaluates on the host with one .item() per boundary in every layer.
 * positions: i64 [T].  Outputs (caller-owned scratch, see mes_varlen_workspace_size):
 *   workspace: opaque buffer of mes_varlen_workspace_size(T) bytes, 256-byte aligned,
 *   holding cu_seqlens (i32 [T+1]), the sequence count and the (sequence, query-tile)
 *   work list consumed by mes_varlen_attention.
 * ------------------------------------------------------------------------------- */
int64_t mes_varlen_workspace_size(int64_t T);
int mes_varlen_schedule(const int64_t* positions, int64_t T, void* workspace, void* stream);

/* Copies cu_seqlens (i32 [num_seqs+1]) out of a scheduled workspace into `cu_seqlens`
 * (device, capacity T+1) and the count into `num_seqs` (device i32 [1]). */
int mes_varlen_cu_seqlens(const void* workspace, int64_t T, int32_t* cu_seqlens,
                          int32_t* num_seqs, void* stream);

/* ---------------------------------------------------------------------------------
 * Varlen causal GQA prefill attention on tcgen05/TMEM.
 * out[t, h*D:(h+1)*D] = softmax_causal(q_h k_g^T * scale) v_g within t's sequence,
 * g = h / (Hq / Hkv).  Replaces FlashAttention.forward / FlashInferAttention.forward
 * (layers/attention/flashattention.py:19-48, layers/attention/flashinfer.py:55-101).
 * qkv: bf16 [T, (Hq + 2*Hkv) * D] (pitch `ld` elements, ld % 8 == 0, 16-byte aligned);
 * out: bf16 [T, Hq * D]; D == 128; workspace from mes_varlen_schedule on the same
 * positions.
 * ------------------------------------------------------------------------------- */
int mes_varlen_attention(const void* qkv, int64_t ld, void* out, const void* workspace,
                         int64_t T, int Hq, int Hkv, int D, float scale, void* stream);

/* ---------------------------------------------------------------------------------
 * The same schedule + attention for callers that cannot allocate device memory (an FFI
 * caller that only holds the buffers its runtime handed over, or a serving process whose
 * device memory is fixed in advance by its own pool).  No counterpart in the reference.
 * The workspace is a fixed array inside this library, on every device that loads it,
 * sized for at most mes_varlen_attention_noalloc_max_tokens() tokens (131072, ~1.5 MiB);
 * larger T returns MES_ERR_INVALID.  Nothing is allocated.  The first call in each CUDA
 * context of a device (and the first after the device's current context changed, e.g.
 * after cudaDeviceReset) looks up the array's device address: make that call before any
 * stream capture.  Every call on a device shares the array: calls whose GPU work overlaps
 * race.
 * positions: i64 [T]; qkv, out, D, scale as for mes_varlen_attention.
 * ------------------------------------------------------------------------------- */
int64_t mes_varlen_attention_noalloc_max_tokens(void);
int mes_varlen_attention_noalloc(const int64_t* positions, const void* qkv, int64_t ld,
                                 void* out, int64_t T, int Hq, int Hkv, int D, float scale,
                                 void* stream);

/* ---------------------------------------------------------------------------------
 * Last-token pooling + L2 normalisation.  out[b, :] = x / max(||x||_2, 1e-12),
 * x = hidden[idx[b], :] (fp32 math and output).
 * Replaces the post-process of GPUWorker._inference_worker (core/gpu_worker.py:252-261)
 * and ultils/pool.py:4-9.
 * hidden: bf16 [T, H]; idx: i64 [B]; out: f32 [B, H]; H % 8 == 0.
 * ------------------------------------------------------------------------------- */
int mes_last_token_l2(const void* hidden, int64_t T, int64_t H, const int64_t* idx,
                      int64_t B, float* out, void* stream);

/* ---------------------------------------------------------------------------------
 * AWQ int4 weights.  Checkpoint format (AutoAWQ GEMM layout): qweight i32 [K, N/8] with
 * nibble i of word (k, j) = code of column 8j + {0,2,4,6,1,3,5,7}[i]; qzeros i32
 * [K/G, N/8] packed the same way; scales f16 [K/G, N]; group size G = 128.
 * Dequantised value: w[k, n] = (q - z) * s, exact in fp32, rounded once to bf16 (RNE).
 * The reference holds dense weights and calls F.linear (layers/linear.py:54,86,179);
 * these entry points replace that GEMM for QKVParallelLinear, MergedColumnParallelLinear
 * and RowParallelLinear (layers/linear.py:90-180).
 * ------------------------------------------------------------------------------- */

/* Repacks a checkpoint qweight [K, N/8] into the kernel layout i32 [K/8, N] (the same
 * nibble interleave applied along K).  Lossless; run once at load time.
 * K % 128 == 0, N % 8 == 0. */
int mes_awq_repack(const int32_t* qweight, int64_t K, int64_t N, int32_t* qweight_mes,
                   void* stream);

/* Dequantises the kernel layout to bf16 W^T [N, K] (row n = output feature n) using the
 * same arithmetic as the GEMM.  For verification. */
int mes_awq_dequant(const int32_t* qweight_mes, const int32_t* qzeros, const void* scales,
                    int64_t K, int64_t N, int group_size, void* w_out, void* stream);

/* Y[M, N] = X[M, K] * W[K, N] (+ bias[N]), W from AWQ (kernel layout), fp32 accumulate
 * on tcgen05, bf16 output.  X: bf16 [M, K] (pitch ldx elements); Y: bf16 [M, N] (pitch
 * ldy); bias: bf16 [N] or NULL; scales: f16 [K/G, N]; qzeros: i32 [K/G, N/8].
 * Requirements: N % 128 == 0, K % 128 == 0, group_size == 128, ldx/ldy % 8 == 0,
 * X, Y, qweight_mes, qzeros and scales 16-byte aligned.  M may be any value >= 0. */
int mes_awq_gemm(const void* X, int64_t ldx, const int32_t* qweight_mes,
                 const int32_t* qzeros, const void* scales, const void* bias, void* Y,
                 int64_t ldy, int64_t M, int64_t N, int64_t K, int group_size, void* stream);

/* Gate/up projection fused with SiLU-and-mul: Y[M, N/2] = bf16(silu(X Wg) * (X Wu)), fp32
 * math on the accumulators.  Replaces MergedColumnParallelLinear.forward followed by
 * SiluAndMul.forward (layers/linear.py:90-107, layers/activation.py:12-14, composed at
 * models/qwen2.py:113-117).  The weight's N = 2I columns must be interleaved in blocks of
 * 16: columns [32b, 32b+16) hold gate features 16b.., columns [32b+16, 32b+32) the up
 * features 16b..; output column 16b + j = silu(gate_{16b+j}) * up_{16b+j}.  qzeros /
 * scales are permuted the same way.  N % 128 == 0, ldy >= N/2. */
int mes_awq_gemm_silu(const void* X, int64_t ldx, const int32_t* qweight_mes,
                      const int32_t* qzeros, const void* scales, void* Y, int64_t ldy, int64_t M,
                      int64_t N, int64_t K, int group_size, void* stream);

/* Same product accumulated into a f32 residual stream: R[M, N] += X * W (+ bias), pitch ldr
 * elements.  This is RowParallelLinear.forward (layers/linear.py:176-180) at tp == 1 fused
 * with the residual add of the following RMSNorm.add_rms_forward (layers/layernorm.py:36),
 * without rounding the projection output to bf16 first. */
int mes_awq_gemm_residual(const void* X, int64_t ldx, const int32_t* qweight_mes,
                          const int32_t* qzeros, const void* scales, const void* bias, float* R,
                          int64_t ldr, int64_t M, int64_t N, int64_t K, int group_size,
                          void* stream);

/* The three GEMMs above with a caller-provided workspace, selected by `epilogue`:
 * 0 = mes_awq_gemm (Y bf16 [M, N]), 1 = mes_awq_gemm_residual (Y = R, f32 [M, N], +=),
 * 2 = mes_awq_gemm_silu (Y bf16 [M, N/2], bias must be NULL).  Same computation and
 * requirements; the same three projections of layers/linear.py:90-180 are replaced.
 * With a workspace of at least mes_awq_gemm_workspace_size(M, N, K) bytes (16-byte
 * aligned), large batches first dequantise the weights once into a bf16 panel W^T [N, K]
 * held there (same exact dequantisation) and then run the tensor-core mainloop on that
 * panel, instead of dequantising again in every token tile.  Batches of 257 to 1024
 * tokens need no workspace (the size is 0): they run the dequantising CTA-pair kernel (as
 * do smaller batches too wide for the one-tile-per-CTA kernel),
 * whose rows equal the panel path's bit for bit.  A NULL or smaller workspace otherwise
 * runs the fused kernels of the three entry points above.  The workspace is scratch:
 * its contents are undefined after the call. */
int64_t mes_awq_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
int mes_awq_gemm_ws(int epilogue, const void* X, int64_t ldx, const int32_t* qweight_mes,
                    const int32_t* qzeros, const void* scales, const void* bias, void* Y,
                    int64_t ldy, int64_t M, int64_t N, int64_t K, int group_size,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* Weight panels for mes_awq_gemm_on_panel: panel i = bf16 W^T [N[i], K[i]] (row n = output
 * feature n, K contiguous, 16-byte aligned) of the kernel-layout AWQ tensors qweight_mes[i],
 * qzeros[i], scales[i], with the GEMM's exact dequantisation.  1 <= count <= 8; the pointer
 * and size arrays are host memory, the tensors device memory.  One launch builds all of
 * them - e.g. the four projections of a decoder layer, shared by both tensor-parallel
 * micro-batches.  Part of the same replacement of the dense F.linear of
 * layers/linear.py:54,86,179 as mes_awq_gemm. */
int mes_awq_panels(int count, const int32_t* const* qweight_mes, const int32_t* const* qzeros,
                   const void* const* scales, const int64_t* K, const int64_t* N,
                   void* const* panels, void* stream);

/* The GEMM of mes_awq_gemm_ws (same `epilogue` codes, Y and bias conventions) with its
 * weights given as a prepared panel (mes_awq_panels) instead of AWQ tensors.  Only for
 * shapes that take the panel path: mes_awq_gemm_workspace_size(M, N, K) > 0 (M > 1024,
 * N % 256 == 0); otherwise MES_ERR_INVALID.  Replaces the same projections
 * (layers/linear.py:90-180). */
int mes_awq_gemm_on_panel(int epilogue, const void* X, int64_t ldx, const void* panel,
                          const void* bias, void* Y, int64_t ldy, int64_t M, int64_t N,
                          int64_t K, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MES_B200_H_ */
