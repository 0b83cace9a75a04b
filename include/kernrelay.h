/*
 * KernRelay C ABI, B200 build (libkernrelay.so for sm_100a).
 *
 * The six entry points, their argument meaning, the caller-owned JSON output
 * buffer and the error convention are those of the reference library
 * (include/kernrelay.h:11-69 of KernRelay 0.3):
 *   - return 0 on success; non-zero on failure, with out = {"error":"..."}
 *     (qwen_main.cpp:2247-2252); C++ exceptions never cross the ABI;
 *   - every string argument is borrowed for the duration of the call;
 *   - device memory, streams, NCCL communicators and peer mappings are created
 *     and destroyed inside the call.
 * B200 differences are additive: modes "tp{k}" / "tp{k}_split" for k in
 * {1,2,4,8} (devices dev0, dev0+1, ... unless KR_TP_DEVICES="a,b,..." is set),
 * and extra JSON fields (status words, k, per-stage device times).
 */
#ifndef KERNRELAY_H
#define KERNRELAY_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Static version string; the caller must not free it.
 * Replaces kr_version (exec/kr_api.cpp:9-12). */
const char *kr_version(void);

/* Run a KernRelay schedule.json (generic DAG executor).
 * Replaces kr_plan_run (include/kernrelay.h:26-27, exec/kr_api.cpp:23-46,
 * exec/exec_main.cpp RunPlanCli).  devices: "" / NULL = 0..nranks-1, else exactly
 * nranks comma-separated ids.  mode: direct | graph | graph_per_stream |
 * graph_segment.  Writes the result JSON {dag, group, nranks, iters, warmup, p50_us,
 * gate_timeouts, checksum, ok, times_us, ... device_p50_us, node_checksums} to
 * out_json and prints it.  Returns 0, 2 on NULL schedule_json/out_json (as the
 * reference does), 1 on any other failure with {"error": "..."} in out_json. */
int kr_plan_run(const char *schedule_json, int iters, int warmup, const char *devices,
                const char *mode, const char *out_json);

/* Single-device Qwen prefill.  mode: serial | serial_fused | serial_graph |
 * graph_whole | relay_event | relay_flag | relay_flag_graph.
 * Replaces kr_qwen_run (include/kernrelay.h:36-37, qwen_main.cpp:2287-2314). */
int kr_qwen_run(const char *model_dir, const char *mode, int seq, int device, int warmup,
                int iters, char *out, size_t out_cap);

/* Two-stage pipeline-parallel prefill (PP=2).  mode: "pp" | "pp1" (requests overlap
 * across the stages) | "pp_serial" | "pp1_serial" (stage 0 starts request r after
 * stage 1 finished r-1).  Stage 0 on dev0 runs layers [0, L/2), stage 1 on dev1
 * layers [L/2, L) and the logits; requests 1..8.  Result JSON: mode (pp_pipeline |
 * pp_serial), seq, requests, devices, layers, wall_best_us, wall_typical_us,
 * wall_samples_us, stages[2] (stage 1 carries argmax / maxdiff).
 * Replaces kr_qwen_pp_run (include/kernrelay.h:45-47, qwen_main.cpp:1993-2146). */
int kr_qwen_pp_run(const char *model_dir, const char *mode, int seq, int dev0, int dev1,
                   int requests, int warmup, int iters, char *out, size_t out_cap);

/* Tensor-parallel-MLP prefill: attention replicated, gate/up column-sharded,
 * down row-sharded, one reduction of the down partial sums per layer.
 *   "tp2"       unsplit down -> NCCL AllReduce -> Add+RMSNorm (baseline)
 *   "tp2_split" down in `tiles` row tiles; each tile's partial sums are pushed
 *               to their owners over NVLink, reduced, all-gathered and
 *               Add+RMSNormed as soon as the tile is released (device flags)
 *   "tp{k}", "tp{k}_split" with k in {1,2,4,8}: same on k devices.
 * tiles in 1..8, seq % tiles == 0.
 * Replaces kr_qwen_tp_run (include/kernrelay.h:57-59, qwen_main.cpp:2225-2254). */
int kr_qwen_tp_run(const char *model_dir, const char *mode, int seq, int dev0, int dev1,
                   int tiles, int warmup, int iters, char *out, size_t out_cap);

/* Per-op k-granularity profile: spec_json = {"cases":[{"op":..,"k":..},..]};
 * ops as in the reference (matmul_q/k/v/o/gate/up/down/lm, add, rmsnorm,
 * add_rmsnorm, rope, silu, mul, embedding, attention).
 * Replaces kr_qwen_profile_many (include/kernrelay.h:68-69, qwen_main.cpp:1535-1783). */
int kr_qwen_profile_many(const char *model_dir, const char *spec_json, int seq, int device,
                         char *out, size_t out_cap);

#ifdef __cplusplus
}
#endif

#endif /* KERNRELAY_H */
