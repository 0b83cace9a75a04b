// Model directory (manifest.json + weights.bin + ids.bin [+ ref files]) and the
// per-rank prefill engine.  The directory format is the reference's
// (scripts/export_model.py:142-223, read by qwen_main.cpp:377-450); the B200
// build additionally accepts tensors marked {"synth": {...}} in the manifest,
// which are generated on the device instead of being read from weights.bin.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "relay.cuh"
#include "tile_sched.h"

namespace krb {

struct ModelCfg {
  std::string arch;
  int H = 0, I = 0, L = 0, HQ = 0, HKV = 0, D = 0, V = 0;
  double eps = 1e-6;
  bool qk_norm = false;
  bool bias = true;
  bool tied = true;
  double theta = 1e6;
  int seq = 0;
  int max_pos = 4096;
  uint64_t seed = 1234;
};

struct TensorSpec {
  std::vector<int64_t> shape;
  size_t offset = 0, bytes = 0;
  bool synth = false;
  std::string kind;    // "normal" | "const" | "transpose_of" (another tensor, transposed)
  double std_ = 0.02;
  double value = 1.0;   // const fill value
  double mean = 0.0;    // normal mean
  uint64_t seed = 0;
  std::string alias;
  size_t numel() const {
    size_t n = 1;
    for (auto d : shape) n *= size_t(d);
    return n;
  }
};

struct Manifest {
  std::string dir;
  ModelCfg cfg;
  std::map<std::string, TensorSpec> tensors;
  bool has(const std::string &n) const { return tensors.count(n) != 0; }
  const TensorSpec &at(const std::string &n) const;
};

Manifest load_manifest(const std::string &dir);

// Execution mode of one engine.
struct Mode {
  std::string name;
  int world = 1;        // TP degree k
  bool tp = false;      // tp* modes (MLP sharded, reduction per layer)
  bool split = false;   // row-tile relay (fused kernel) instead of GEMM + AllReduce
  bool graph = false;   // capture the prefill into a CUDA graph and replay it
  bool fused = true;    // Add+RMSNorm fused (serial = unfused add then norm)
  bool pp = false;      // pp*: layer pipeline over two devices (one stage per engine)
  bool pp_pipeline = false;  // pp / pp1: requests overlap across the stages
  static Mode parse(const std::string &name);
};

struct EngineOpts {
  std::string model_dir;
  std::string mode = "serial";
  int seq = 2048;
  int rank = 0;
  int world = 1;
  int device = 0;
  int tiles = 4;
  int lm_rows = -1;   // -1: all S rows (reference); 1: last row only
  int pp_stage = 0;   // pp modes: this engine's stage and the number of stages
  int pp_stages = 1;
  // Isolated TP-MLP micro-DAG (no model directory): per rank, X_r [seq, md_I/world]
  // ~ N(0,1) and W_r [md_I/world, md_H] ~ N(0,0.02) (seed md_seed + rank), residual
  // R [seq, md_H] ~ N(0,1) (seed md_seed), gamma = 1; one step = down GEMM ->
  // reduction over the ranks -> Add+RMSNorm, by the relay (split modes) or GEMM +
  // NCCL AllReduce + Add+RMSNorm (tp modes).  Tensor names: microdag.X,
  // microdag.W_down, microdag.R (the synthetic generator of synth.cuh).
  bool microdag = false;
  int md_H = 0, md_I = 0;
  uint64_t md_seed = 1234;
};

// Per-stage device time accumulated by an instrumented run (microseconds).
struct StageTimes {
  double embed = 0, qkv = 0, rope = 0, attn = 0, o = 0, addnorm = 0, gateup = 0, down = 0,
         allreduce = 0, addnorm2 = 0, relay = 0, lm_head = 0, total = 0;
};

class Engine {
 public:
  explicit Engine(const EngineOpts &o);
  ~Engine();
  Engine(const Engine &) = delete;
  Engine &operator=(const Engine &) = delete;

  const ModelCfg &cfg() const { return m_.cfg; }
  const Mode &mode() const { return mode_; }
  int rank() const { return opts_.rank; }
  int world() const { return opts_.world; }
  int device() const { return opts_.device; }
  cudaStream_t stream() const { return stream_; }

  // symmetric relay region (tp split modes); null otherwise
  void *sym_base() const { return sym_; }
  size_t sym_bytes() const { return sym_layout_.bytes; }
  void set_peers(const std::vector<void *> &bases);  // index = rank, own entry = sym_base()
  void set_nccl(ncclComm_t comm) { nccl_ = comm; }

  // one prefill on the engine stream (asynchronous)
  void enqueue();
  // one prefill with the host-side copies a caller pays: ids from pinned host
  // memory to the device, last-row logits back to the host (fp32)
  void enqueue_host(const int64_t *ids_host, float *last_logits_host);
  void capture_graph();
  void run();  // graph replay if captured, else enqueue()
  void sync();
  uint32_t read_status();
  StageTimes instrumented_run();

  // correctness: compare the last-row logits with ref_last_logits.bin / ref.json
  struct Verdict {
    int argmax = -1, ref_argmax = -1;
    double maxdiff = 0, abs_mean = 0;
    bool has_ref = false;
  };
  Verdict verify();
  std::vector<float> last_logits();
  // device pointers for tests / profiling
  const float *hidden_ptr() const;  // fp32 residual stream after the last layer (hf)
  int lm_rows() const { return lm_rows_; }
  // kernels of this library launched by the last enqueue (one prefill)
  int launches() const { return launches_; }
  // layers [layer_begin, layer_end) run on this engine (all of them except in pp modes)
  int layer_begin() const { return layer_begin_; }
  int layer_end() const { return layer_end_; }
  // this engine produces the logits: TP rank 0 of the last pipeline stage
  bool has_logits() const { return !opts_.microdag && opts_.rank == 0 && layer_end_ == m_.cfg.L; }
  bool microdag() const { return opts_.microdag; }
  // final normed rows xf [S, H] fp16 (the micro-DAG's x output)
  const __half *final_x_ptr() const { return xf_; }
  // pp: enqueue this stage's part of one prefill; a later stage takes the fp32
  // residual stream [S, H] of the previous stage from `h_in` (device memory)
  void enqueue_stage(const float *h_in);
  const float *residual_out() const { return h0_; }
  const char *relay_kind() const {
    return mode_.split ? (relay_direct_ ? "direct" : "rsag") : "none";
  }
  // per-op k-slice timing table (kr_qwen_profile_many)
  std::string profile_many(const std::string &spec_path);
  // dump the residual stream after every layer into host memory on the next run
  void set_layer_dump(bool on);
  std::vector<float> layer_hidden(int l);  // fp32 residual [S, H]

 private:
  void load_weights();
  void alloc_activations();
  void fetch(const std::string &name, __nv_bfloat16 *staging);
  void layer(int l, StageTimes *st);
  // layer l's down projection, reduction over the ranks and Add+RMSNorm (the tile loop
  // of qwen_main.cpp:1274-1302, or its unsplit form)
  void down_stage(int l, StageTimes *st, const __nv_bfloat16 *gamma, float *sum_out,
                  __half *x_out, bool do_norm);
  void load_microdag();
  void microdag_enqueue(StageTimes *st);
  void prologue(StageTimes *st);
  void epilogue(StageTimes *st);
  void add_norm(const float *res, const __half *delta, const __nv_bfloat16 *gamma, __half *y,
                float *sum);

  EngineOpts opts_;
  Manifest m_;
  Mode mode_;
  int layer_begin_ = 0, layer_end_ = 0;
  bool fuse_rope_ = false;  // QK-norm + RoPE in the QKV GEMM epilogue
  // tp modes: o_proj, the residual add and ln2 in one relay kernel at k = 1 (its own
  // counters and run epoch in oflags_, o_tiles_ row tiles); KRB_FUSE_OPROJ=0 keeps the
  // o_proj GEMM + Add+RMSNorm pair
  bool fuse_oproj_ = false;
  int o_tiles_ = 0;
  SymLayout oflags_layout_{};
  void *oflags_ = nullptr;
  int Iloc_ = 0, nqkv_ = 0, bn_gu_ = 256, bn_down_ = 256, gu_rows_ = 0;
  int lm_rows_ = 0;
  int launches_ = 0;
  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t graph_ = nullptr;
  ncclComm_t nccl_ = nullptr;

  // weights: the GEMM operands in fp16 (converted exactly from the bf16 checkpoint at
  // load); biases, norm weights, rope tables and the embedding table stay bf16
  struct LayerW {
    __half *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
    __nv_bfloat16 *bqkv = nullptr, *ln1 = nullptr, *ln2 = nullptr, *qn = nullptr, *kn = nullptr;
  };
  std::vector<LayerW> lw_;
  __nv_bfloat16 *embed_ = nullptr, *final_norm_ = nullptr, *cos_ = nullptr, *sin_ = nullptr,
                *md_gamma_ = nullptr;
  __half *wlm_ = nullptr;
  std::vector<void *> allocs_;
  void *weight_map_ = nullptr;
  size_t weight_map_bytes_ = 0;
  std::string weight_map_dir_;

  // activations
  // residual stream in fp32 (h0: layer input, h1: after attention, hf: final);
  // everything the GEMMs read or write is fp16 (8x finer rounding than bf16; the
  // per-layer error against the fp32 oracle of a 28-layer 7B model stays near 1e-3
  // per layer instead of growing past 1e-2)
  float *h0_ = nullptr, *h1_ = nullptr, *hf_ = nullptr;
  float *delta_ = nullptr;  // fp32 o_proj / down output before the residual add
  __half *x_ = nullptr, *qkv_ = nullptr, *attn_ = nullptr, *o_ = nullptr, *act_ = nullptr,
         *down_ = nullptr, *red_ = nullptr, *xf_ = nullptr, *logits_ = nullptr;
  int64_t *ids_ = nullptr;
  uint32_t *status_ = nullptr;
  float *last_f32_ = nullptr;
  float *dump_ = nullptr;  // [L, S, H] fp32 when layer dumps are on
  __half *vt_ = nullptr;  // fp16 V^T [HKV*D, ldvt_] for the tcgen05 attention
  long ldvt_ = 0;

  // relay
  SymLayout sym_layout_{};
  void *sym_ = nullptr;
  std::vector<void *> peers_;
  int relay_direct_ = 0;  // 1: direct all-pull relay, 0: reduce-scatter + all-gather
  int relay_ready_order_ = 0;  // rsag: fixed pipeline order (KRB_RELAY_ORDER=ready: readiness)
  int nseg_ = 0;
  uint64_t flag_timeout_ns_ = 2000000000ull;
  unsigned long long *trace_ = nullptr;  // relay phase trace (KRB_RELAY_TRACE=1)
 public:
  // copy of the relay trace of the last relay launch: [grid][kTraceSlots] ns
  std::vector<unsigned long long> relay_trace();
 private:

  void *alloc(size_t bytes);
};

// relay launcher (relay.cu); T = __half (every rank count) or __nv_bfloat16 (one rank).
// The 2-byte buffers of RelayArgs (partials, reduced rows, x_out) hold T.
template <typename T>
void relay_down_layer(const T *act, long lda, const T *w_down, long ldb, int bn,
                      const RelayArgs &ra, cudaStream_t stream);
// the relay GEMM's tile schedule for `grid` CTAs (row tile t = band t; cta_group 2: CTA
// pairs on 256-row tiles), and whether the relay runs its GEMM on CTA pairs
TileSched relay_tile_sched(int S, int H, int T, int bn, int grid, int cta_group);
bool relay_uses_pairs(int S, int T, int bn);

// device-side synthesis / fill (synth.cu)
void synth_normal_device(__nv_bfloat16 *dst, size_t n, uint64_t key, double std_, double mean,
                         cudaStream_t stream);
void fill_const_device(__nv_bfloat16 *dst, size_t n, float value, cudaStream_t stream);
void bump_epoch(uint32_t *epoch, cudaStream_t stream);
// this device's static relay scratch (kRelayNoAllocScratchBytes); the first call
// per device looks the symbol up
uint8_t *relay_noalloc_scratch();
void bf16_row_to_f32(const __nv_bfloat16 *src, float *dst, int n, cudaStream_t stream);

}  // namespace krb
