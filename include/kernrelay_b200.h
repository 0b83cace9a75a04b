/*
 * B200 extensions of the KernRelay C ABI (libkernrelay.so, sm_100a).
 *
 * kernrelay.h keeps the reference's six entry points.  The reference runs all
 * TP ranks as threads of one process (qwen_main.cpp:1871-1989); a B200 box is
 * normally driven one process per GPU, so this header adds a per-rank engine
 * whose ranks exchange CUDA IPC handles of their relay regions (and, for the
 * NCCL "tp" baseline, an ncclUniqueId) through any host channel, e.g.
 * torch.distributed.  It also exposes every hot-path kernel as a stand-alone
 * op on caller-owned device memory, which the parity tests and the profiler
 * call directly.
 *
 * Conventions: return 0 on success; non-zero on failure, with the message
 * available from krb_last_error() (thread-local).  Device pointers are raw
 * addresses in the current device's address space; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  All bf16 tensors are
 * row-major with the stated leading dimensions (elements).
 */
#ifndef KERNRELAY_B200_H
#define KERNRELAY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the last failing krb_* call on this thread ("" if none). */
const char *krb_last_error(void);

/* Number of visible CUDA devices (0 without a GPU; never fails). */
int krb_device_count(void);

/* ---------------------------------------------------------------- host synthesis
 * Element values of a synthetic tensor (manifest entry {"synth": {"kind":
 * "normal", "std": s, "mean": m, "seed": seed}}), elements [offset, offset+n) of the
 * tensor's flat reference layout, as raw bf16 bits.  CPU only; the device
 * loader produces bit-identical values.  (No reference counterpart: the
 * reference exports real checkpoints, scripts/export_model.py:159-169.) */
int krb_synth_normal_host(const char *name, uint64_t seed, double std_, double mean,
                          uint64_t offset, uint64_t n, uint16_t *out);

/* ---------------------------------------------------------------- stand-alone ops */
/* C[M,N] = A[M,K] . B[N,K]^T (+ bias[N]); tcgen05 GEMM.  bn = UMMA N tile
 * (128, 224, 256) or 0 for automatic.  Replaces aclnnMatmul (+ aclnnAdd bias),
 * qwen_main.cpp:499-512, :1336-1344. */
int krb_gemm_bf16(const void *A, long lda, const void *B, long ldb, void *C, long ldc,
                  const void *bias, int M, int N, int K, int bn, void *stream);

/* Fused QKV projection: C[M,(HQ+2HKV)D] = A . B^T + bias, then per q / k head an
 * optional RMSNorm over D (q_norm / k_norm; Qwen3) and rotate-half RoPE with the bf16
 * cos / sin tables [max_pos, D] at position = row, in the GEMM epilogue; v heads get the
 * bias only.  D in {64, 128}.  Replaces EmitQkv + EmitQkNorm + aclnnApplyRotaryPosEmb
 * (qwen_main.cpp:1336-1357, 567-582) as one kernel. *  vt (optional, fp16 [HKV*D][ldvt >= M]): the v heads also written transposed,
 *  vt[(c - (HQ+HKV)*D) * ldvt + row] = fp16(bf16 value) -- the attention's V^T. */
int krb_gemm_qkv_rope_bf16(const void *A, long lda, const void *B, long ldb, void *C, long ldc,
                           const void *bias, int M, int K, int HQ, int HKV, int D,
                           const void *cos_tab, const void *sin_tab, const void *q_norm,
                           const void *k_norm, float eps, void *vt, long ldvt, void *stream);

/* out[M,N] = A[M,K] . B[N,K]^T in fp32 (unrounded; row pitch ld) -- the o_proj and
 * single-device down_proj form whose output feeds the fp32 residual stream. */
int krb_gemm_f32out(const void *A, long lda, const void *B, long ldb, float *out, long ld, int M,
                    int N, int K, int bn, void *stream);

/* act[M, n_out] = silu(A.Bg^T) * (A.Bu^T) where Bgu interleaves gate and up
 * rows in blocks of bn: rows [b*bn, b*bn+bn/2) = gate rows [b*bn/2, (b+1)*bn/2),
 * rows [b*bn+bn/2, (b+1)*bn) = the matching up rows (bn = 128, 192 or 256).
 * Replaces the gate/up aclnnMatmul + aclnnSilu + aclnnMul, qwen_main.cpp:1267-1271. */
int krb_gemm_silu_bf16(const void *A, long lda, const void *Bgu, long ldb, void *act, long ldact,
                       int M, int n_out, int K, int bn, void *stream);

/* y = x * rsqrt(mean(x^2) + eps) * gamma, rows of H.  Replaces aclnnRmsNorm
 * (qwen_main.cpp:531-546); rstd may be NULL. */
int krb_rmsnorm_bf16(const void *x, const void *gamma, void *y, float *rstd, int rows, int H,
                     float eps, void *stream);

/* sum = bf16(a + b); y = RMSNorm(sum) * gamma.  Replaces aclnnAddRmsNorm
 * (qwen_main.cpp:548-565); sum and rstd may be NULL. */
int krb_add_rmsnorm_bf16(const void *a, const void *b, const void *gamma, void *y, float *rstd,
                         void *sum, int rows, int H, float eps, void *stream);

/* Residual-stream form used by the engine: sum = res + delta in fp32 (res and
 * sum fp32 [rows, H], delta bf16 or NULL), y = RMSNorm(sum) * gamma (bf16). */
int krb_add_rmsnorm_res_f32(const float *res, const void *delta, const void *gamma, void *y,
                            float *sum, int rows, int H, float eps, void *stream);

/* out[s,:] = table[ids[s],:]; ids outside [0,V) produce zero rows and set
 * bit 7 of *status (may be NULL).  Replaces aclnnEmbedding (qwen_main.cpp:646-659). */
int krb_embed_bf16(const int64_t *ids, const void *table, void *out, int S, int H, int V,
                   uint32_t *status, void *stream);

/* In place on qkv [S, (HQ+2*HKV)*D]: optional per-head RMSNorm over D of the
 * q and k heads (q_norm/k_norm NULL to skip), then rotate-half RoPE with
 * cos/sin [>=S, D].  Replaces EmitQkNorm + aclnnApplyRotaryPosEmb
 * (qwen_main.cpp:1346-1357, :567-582). */
int krb_qk_norm_rope_bf16(void *qkv, int S, int HQ, int HKV, int D, const void *cos_tab,
                          const void *sin_tab, const void *q_norm, const void *k_norm, float eps,
                          void *stream);

/* out[S, HQ*D] = causal GQA attention of the q/k/v heads of qkv with the given
 * scale.  impl: 0 = automatic (tcgen05/TMEM kernel for D = 128, else mma.sync),
 * 1 = mma.sync kernel, 2 = tcgen05 kernel (D = 128 only; uses a V^T scratch of
 * HKV*D*S bf16 allocated and freed stream-ordered on `stream`).  Wait timeouts
 * set bits in *status (may be NULL).  Replaces aclnnFlashAttentionScore
 * (qwen_main.cpp:591-614). */
int krb_attention_prefill_bf16(const void *qkv, void *out, int S, int HQ, int HKV, int D,
                               float scale, int impl, uint32_t *status, void *stream);

/* Fused down-GEMM + row-tile relay + Add+RMSNorm on ONE device (tp degree 1):
 *   down = act[S,K] . w_down[H,K]^T (bf16 partial), released to the consumer
 *   warps tile by tile through device counters; sum = resid + down (resid and
 *   sum fp32 [S,H]); x = RMSNorm(sum)*gamma (bf16).
 * The relay scratch (partial rows, gathered rows, counters: about 4*S*H bytes)
 * is allocated by this call with cudaMalloc and freed before it returns, after
 * synchronising `stream`.  Replaces the tp_split tile loop of qwen_main.cpp:1274-1302
 * for k = 1. */
int krb_relay_down_single(const void *act, const void *w_down, const void *resid,
                          const void *gamma, void *sum_out, void *x_out, int S, int H, int K,
                          int tiles, float eps, int bn, uint32_t *status, void *stream);

/* Allocation-free form of krb_relay_down_single (same arguments, same results; no
 * counterpart in the reference).  For callers that must not allocate device memory
 * inside the call: a serving engine that reserved nearly all of HBM up front for
 * its own pools, or a caller with work in flight on other streams, which the
 * implicit device synchronisation of cudaFree would stall.  The relay's flag
 * counters and run epoch live in a static device array of 32 KiB per device
 * ((2 * tiles + 2) * 128 bytes are used, so tiles <= 127; more returns an error).
 * The call zeroes them on `stream`, launches, and returns without synchronising.
 * The first call on a device does its set-up (symbol lookup, kernel attributes)
 * and should come before any stream capture on that device.  The looked-up address
 * is kept for the life of the process: do not reset the device (cudaDeviceReset or
 * a primary-context reset) between calls.  Calls that overlap
 * in time on one device (different streams or threads) share the scratch and
 * race; calls in order on one stream are safe.  k = 1 only, like
 * krb_relay_down_single. */
int krb_relay_down_single_noalloc(const void *act, const void *w_down, const void *resid,
                                  const void *gamma, void *sum_out, void *x_out, int S, int H,
                                  int K, int tiles, float eps, int bn, uint32_t *status,
                                  void *stream);

/* Failure-detection probe: runs the relay kernel as rank 0 of a two-rank job
 * whose peer never participates (its region is a second local allocation that
 * nobody signals).  Rank 0's bounded waits expire after timeout_ms; the kernel
 * records the status bits (bit 3: partials missing, bit 4: all-gather missing)
 * in *status_out and returns with the CUDA context usable.  Allocates and frees
 * its own buffers; synchronises the device.  (The reference's equivalent is the
 * kr_wait_* status word 2 after maxSpins, kernels/kr_wait_aiv.cpp:22-33.) */
int krb_relay_timeout_probe(int S, int H, int K, int tiles, float timeout_ms, uint32_t *status_out);

/* Parse and validate a schedule.json exactly as kr_plan_run does, without a GPU:
 * JSON {dag, group, nranks, nodes, tasks, publishes, lanes, segments,
 * lane_order_acyclic} or {"error": ...} (rc 1) with kr_plan_run's message. */
int krb_plan_check(const char *schedule_json, char *out, size_t cap);

/* Host view of the tp_split relay plan for (S, H, tiles, k, rank, bn): JSON
 * {R, Rk, num_n, rs_expect, ag_expect, nseg, blocks: [[tile, first_owner,
 * last_owner] per 128-row block]} -- the row routing the device epilogue uses
 * and the counter targets the consumer waits for (per layer and run). */
int krb_relay_plan(int S, int H, int tiles, int k, int rank, int bn, char *out, size_t cap);

/* ---------------------------------------------------------------- per-rank engine */
typedef struct krb_engine krb_engine;

/* Load the model directory for (rank, world) on `device` and allocate all
 * buffers.  mode: any kr_qwen_run mode (world 1) or tp{k}[_split][_graph]. */
int krb_engine_create(const char *model_dir, const char *mode, int seq, int rank, int world,
                      int device, int tiles, krb_engine **out);
void krb_engine_destroy(krb_engine *e);

/* An engine for the isolated TP-MLP micro-DAG (the reference's mm -> AllReduce ->
 * AddNorm tile loop, qwen_main.cpp:1274-1302, without the rest of the layer): per
 * rank X_r [seq, intermediate/world] ~ N(0,1) and W_r [intermediate/world, hidden]
 * ~ N(0,0.02) generated with seed + rank, residual R [seq, hidden] ~ N(0,1) with
 * seed, gamma = 1, eps 1e-6.  mode: tp{k} (GEMM -> NCCL AllReduce -> Add+RMSNorm) or
 * tp{k}_split (the fused relay, `tiles` row tiles).  Every engine call below
 * applies; one run is one micro-DAG step and every rank's outputs are read with
 * krb_engine_final_hidden (h = R + sum of the partials, fp32) and krb_engine_final_x
 * (x = RMSNorm(h), bf16). */
int krb_microdag_create(int seq, int hidden, int intermediate, int tiles, int rank, int world,
                        int device, const char *mode, uint64_t seed, krb_engine **out);

/* tp_split: cudaIpcMemHandle_t (64 bytes) of this rank's relay region. */
int krb_engine_ipc_handle(krb_engine *e, void *handle_out, size_t cap);
/* tp_split: map every peer's relay region; handles = world x 64 bytes (own entry ignored). */
int krb_engine_open_peers(krb_engine *e, const void *handles, size_t bytes);
/* tp (NCCL baseline): rank 0 creates the id (128 bytes), every rank joins. */
int krb_nccl_unique_id(void *out, size_t cap);
int krb_engine_init_nccl(krb_engine *e, const void *id, size_t bytes);

/* One process driving k engines (ranks 0..k-1, one device each): enable peer
 * access and wire the relay regions directly (tp_split), or create the NCCL
 * communicators with ncclCommInitAll (tp).  Run the engines from one host
 * thread each (NCCL's rule for one process and several devices). */
int krb_engines_link(krb_engine **engines, int n);
int krb_engines_init_nccl(krb_engine **engines, int n);

int krb_engine_capture(krb_engine *e);          /* capture one prefill into a CUDA graph */
int krb_engine_run(krb_engine *e);              /* enqueue one prefill (async) */
/* ids (pinned host, S int64) -> device, prefill, last-row logits -> host fp32 [V] (rank 0) */
int krb_engine_run_host(krb_engine *e, const int64_t *ids_host, float *logits_host);
int krb_engine_sync(krb_engine *e);
int krb_engine_stream(krb_engine *e, void **stream_out);
int krb_engine_status(krb_engine *e, uint32_t *status_out);
/* one instrumented prefill; JSON {"stage_us":{...},"total_us":...} */
int krb_engine_stage_times(krb_engine *e, char *out, size_t cap);
/* last-row logits vs ref files; JSON {argmax, ref_argmax, maxdiff, abs_mean, has_ref} */
int krb_engine_verify(krb_engine *e, char *out, size_t cap);
int krb_engine_last_logits(krb_engine *e, float *out, int n);
/* copy the fp32 residual stream after the final layer ([S,H], rank 0; every rank of
 * a micro-DAG engine) to host */
int krb_engine_final_hidden(krb_engine *e, float *out, size_t n);
/* copy the final normed rows xf ([S,H] fp16, rank 0; every rank of a micro-DAG
 * engine) to host */
int krb_engine_final_x(krb_engine *e, uint16_t *out, size_t n);
/* keep a copy of the residual stream after every layer of the next runs
 * (test-sized models: L*S*H*2 bytes of device memory) */
int krb_engine_layer_dump(krb_engine *e, int on);
/* fp32 [S, H] residual after `layer` (the last layer's entry is the pre-norm
 * final hidden state, rank 0 only) */
int krb_engine_layer_hidden(krb_engine *e, int layer, float *out, size_t n);
/* Relay phase trace of the last relay launch (engine built with KRB_RELAY_TRACE=1):
 * per CTA kTraceSlots globaltimer stamps (ns) -- start, GEMM epilogue done, relay
 * done, then per row tile: partials arrived, reduced+pushed, all-gather arrived,
 * Add+RMSNorm done.  *written = number of values (0 when tracing is off). */
int krb_engine_relay_trace(krb_engine *e, unsigned long long *out, size_t n, size_t *written);
/* describe the engine: JSON {H, I, L, V, seq, world, rank, lm_rows, bn_*} */
int krb_engine_info(krb_engine *e, char *out, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* KERNRELAY_B200_H */
