// Per-rank Qwen prefill engine over one CUDA stream.
//
// Program per layer (reference op order: BuildSerial qwen_main.cpp:925-992 and
// BuildTP :1220-1309; every reference op maps onto one of our kernels):
//   qkv   = x . [Wq;Wk;Wv]^T + [bq;bk;bv]       tcgen05 GEMM, bias epilogue   (EmitQkv :1336-1344)
//   q,k   = QKNorm? -> RoPE (in place)           qk_norm_rope                 (EmitQkNorm :1346-1357, Rope :567-582)
//   attn  = causal GQA attention                 attention_prefill            (FlashN :591-614)
//   o     = attn . Wo^T                          tcgen05 GEMM                 (:1262)
//   h1,x  = AddRMSNorm(h0, o, ln2)               add_rmsnorm                  (:1264-1265)
//   act   = silu(x Wg^T) * (x Wu^T)               tcgen05 GEMM, SiLU epilogue  (:1267-1271)
//   tp / single:  down = act . Wd^T -> [NCCL AllReduce] -> h0,x = AddRMSNorm(h1, red, ln1[l+1])
//   tp_split:     relay_down_layer (fused GEMM + push + reduce + all-gather + AddRMSNorm)
// then lm_head = xf . Wlm^T on rank 0 (reference :1305-1307).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>

#include "json_min.hpp"
#include "model.h"
#include "synth.cuh"

namespace krb {

// ------------------------------------------------------------------ manifest
const TensorSpec &Manifest::at(const std::string &n) const {
  auto it = tensors.find(n);
  if (it == tensors.end()) throw std::runtime_error("manifest: missing tensor " + n);
  return it->second;
}

Manifest load_manifest(const std::string &dir) {
  Manifest m;
  m.dir = dir;
  json::Value doc = json::parse_file(dir + "/manifest.json");
  const json::Value &c = doc.at("config");
  ModelCfg &g = m.cfg;
  g.arch = c.string_or("arch", "qwen2.5");
  g.H = int(c.at("hidden_size").num);
  g.I = int(c.at("intermediate_size").num);
  g.L = int(c.at("num_hidden_layers").num);
  g.HQ = int(c.at("num_attention_heads").num);
  g.HKV = int(c.at("num_key_value_heads").num);
  g.V = int(c.at("vocab_size").num);
  g.D = c.has("head_dim") ? int(c.at("head_dim").num) : g.H / g.HQ;
  g.qk_norm = c.bool_or("qk_norm", false);
  g.eps = c.number_or("rms_norm_eps", 1e-6);
  g.tied = c.bool_or("tie_word_embeddings", true);
  g.theta = c.number_or("rope_theta", 1e6);
  g.seq = int(doc.at("seq").num);
  g.max_pos = int(doc.number_or("max_pos", 4096));
  g.seed = uint64_t(doc.number_or("seed", 1234));
  for (const auto &kv : doc.at("tensors").obj) {
    TensorSpec t;
    for (const auto &d : kv.second.at("shape").arr) t.shape.push_back(int64_t(d.num));
    if (kv.second.has("synth")) {
      const json::Value &s = kv.second.at("synth");
      t.synth = true;
      t.kind = s.string_or("kind", "normal");
      t.std_ = s.number_or("std", 0.02);
      t.value = s.number_or("value", 1.0);
      t.mean = s.number_or("mean", 0.0);
      t.seed = uint64_t(s.number_or("seed", double(g.seed)));
      t.alias = s.string_or("of", "");
    } else {
      t.offset = size_t(kv.second.at("offset").num);
      t.bytes = size_t(kv.second.at("bytes").num);
      const std::string dt = kv.second.string_or("dtype", "bfloat16");
      if (dt != "bfloat16") throw std::runtime_error("manifest: " + kv.first + " is not bfloat16");
      if (t.bytes != t.numel() * 2) throw std::runtime_error("manifest: bad byte count " + kv.first);
    }
    m.tensors[kv.first] = t;
  }
  // QKV bias is used when the config says so and the tensors exist (qwen_main.cpp:389-390)
  g.bias = c.bool_or("attention_bias", true) && m.has("L00.q_proj.bias");
  return m;
}

// ------------------------------------------------------------------ modes
Mode Mode::parse(const std::string &name) {
  Mode m;
  m.name = name;
  if (name == "serial") {
    m.fused = false;
  } else if (name == "serial_fused") {
  } else if (name == "serial_graph") {
    m.graph = true;
    m.fused = false;
  } else if (name == "graph_whole") {
    m.graph = true;
  } else if (name == "relay_event" || name == "relay_flag") {
    m.split = true;
  } else if (name == "relay_flag_graph") {
    m.split = true;
    m.graph = true;
  } else if (name == "pp" || name == "pp1" || name == "pp_serial" || name == "pp1_serial") {
    // PP=2 (qwen_main.cpp:1359-1528, 1993-2146): "pp"/"pp1" overlap the requests
    // across the stages, "pp_serial"/"pp1_serial" run them one after another
    m.pp = true;
    m.pp_pipeline = name == "pp" || name == "pp1";
  } else if (name.rfind("tp", 0) == 0) {
    // tp{k}[_split][_graph]; "tp" alone means k=2 as in the reference's tp2
    std::string rest = name.substr(2);
    size_t p = 0;
    while (p < rest.size() && isdigit(static_cast<unsigned char>(rest[p]))) ++p;
    m.world = p ? std::atoi(rest.substr(0, p).c_str()) : 2;
    std::string suf = rest.substr(p);
    m.tp = true;
    if (suf.rfind("_split", 0) == 0) {
      m.split = true;
      suf = suf.substr(6);
    }
    if (suf == "_graph") {
      m.graph = true;
      suf.clear();
    }
    if (!suf.empty()) throw std::runtime_error("unknown mode " + name);
    if (m.world != 1 && m.world != 2 && m.world != 4 && m.world != 8)
      throw std::runtime_error("tp degree must be 1, 2, 4 or 8");
  } else {
    throw std::runtime_error("unknown mode " + name);
  }
  return m;
}

// ------------------------------------------------------------------ engine
void *Engine::alloc(size_t bytes) {
  void *p = nullptr;
  KRB_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
  allocs_.push_back(p);
  return p;
}

static std::string layer_prefix(int l) {
  char b[16];
  std::snprintf(b, sizeof(b), "L%02d.", l);
  return b;
}

Engine::Engine(const EngineOpts &o) : opts_(o) {
  mode_ = Mode::parse(o.mode);
  if (!mode_.tp && opts_.world != 1) throw std::runtime_error("single-device mode with world > 1");
  if (mode_.tp && mode_.world != opts_.world)
    throw std::runtime_error("mode tp degree does not match world size");
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  if (opts_.microdag) {
    // no model directory: one "layer" holding only the down projection
    if (!mode_.tp) throw std::runtime_error("micro-DAG: mode must be tp{k} or tp{k}_split");
    if (opts_.md_H <= 0 || opts_.md_I <= 0) throw std::runtime_error("micro-DAG: bad shape");
    m_.dir.clear();
    ModelCfg &g = m_.cfg;
    g.arch = "tp_mlp_microdag";
    g.H = opts_.md_H;
    g.I = opts_.md_I;
    g.L = 1;
    g.HQ = g.HKV = 1;
    g.D = 128;
    g.V = 0;
    g.eps = 1e-6;
    g.seq = opts_.seq;
    g.max_pos = opts_.seq;
    g.seed = opts_.md_seed;
  } else {
    m_ = load_manifest(opts_.model_dir);
  }
  const ModelCfg &c = m_.cfg;
  if (c.seq != opts_.seq) throw std::runtime_error("manifest seq mismatch");
  if (c.I % opts_.world) throw std::runtime_error("intermediate size not divisible by tp degree");
  if (c.HQ % c.HKV) throw std::runtime_error("heads not divisible by kv heads");
  if (opts_.seq > c.max_pos) throw std::runtime_error("seq exceeds rope table");
  if (opts_.tiles < 1 || opts_.tiles > 8) throw std::runtime_error("tiles must be in 1..8");
  if (opts_.seq % opts_.tiles) throw std::runtime_error("seq % tiles != 0");
  if (const char *e = std::getenv("KRB_FLAG_TIMEOUT_MS"))
    flag_timeout_ns_ = uint64_t(std::max(1.0, std::atof(e)) * 1e6);
  Iloc_ = c.I / opts_.world;
  nqkv_ = (c.HQ + 2 * c.HKV) * c.D;
  layer_begin_ = 0;
  layer_end_ = c.L;
  // fused modes run RoPE (and QK-norm) in the QKV GEMM epilogue; KRB_FUSE_ROPE=0 keeps
  // the separate kernel
  fuse_rope_ = mode_.fused && !(std::getenv("KRB_FUSE_ROPE") && std::getenv("KRB_FUSE_ROPE")[0] == '0');
  if (mode_.pp) {
    // stage s of n runs layers [s*L/n, (s+1)*L/n) (qwen_main.cpp:746-747)
    if (opts_.pp_stages < 2 || opts_.pp_stage < 0 || opts_.pp_stage >= opts_.pp_stages)
      throw std::runtime_error("pp: bad stage");
    layer_begin_ = opts_.pp_stage * c.L / opts_.pp_stages;
    layer_end_ = (opts_.pp_stage + 1) * c.L / opts_.pp_stages;
  }
  const int sms = sm_count(opts_.device);
  bn_gu_ = pick_bn_silu(opts_.seq, Iloc_, sms);
  const int half = bn_gu_ / 2;
  gu_rows_ = ((Iloc_ + half - 1) / half) * bn_gu_;
  bn_down_ = pick_bn_store(opts_.seq, c.H, sms);
  // o_proj + residual + ln2 fused (tp modes, split and NCCL alike, so the two arms keep
  // the same attention block): 4 row tiles when they are whole CTA-pair blocks, else 1
  if (mode_.tp && mode_.fused && !opts_.microdag &&
      !(std::getenv("KRB_FUSE_OPROJ") && std::getenv("KRB_FUSE_OPROJ")[0] == '0')) {
    o_tiles_ = (opts_.seq % (4 * 256) == 0) ? 4 : 1;
    if ((opts_.seq / o_tiles_) % 128 == 0) fuse_oproj_ = true;
  }
  lm_rows_ = opts_.lm_rows > 0 ? std::min(opts_.lm_rows, opts_.seq) : opts_.seq;
  if (const char *e = std::getenv("KRB_LM_ROWS")) {
    const int r = std::atoi(e);
    if (r > 0) lm_rows_ = std::min(r, opts_.seq);
  }
  status_ = static_cast<uint32_t *>(alloc(256));
  KRB_CUDA(cudaMemset(status_, 0, 256));
  if (opts_.microdag) {
    load_microdag();
  } else {
    load_weights();
    alloc_activations();
  }
  if (fuse_oproj_) {
    oflags_layout_ = SymLayout::flags_only(o_tiles_);
    KRB_CUDA(cudaMalloc(&oflags_, oflags_layout_.bytes));
    KRB_CUDA(cudaMemset(oflags_, 0, oflags_layout_.bytes));
  }
  if (mode_.split) {
    const int S = opts_.seq, T = opts_.tiles, k = opts_.world;
    if ((S / T) % 128) throw std::runtime_error("tp_split needs seq/tiles to be a multiple of 128");
    if ((S / T) % k) throw std::runtime_error("tp_split needs seq/tiles divisible by tp degree");
    sym_layout_ = SymLayout::make(S, c.H, T, k);
    KRB_CUDA(cudaMalloc(&sym_, sym_layout_.bytes));
    KRB_CUDA(cudaMemset(sym_, 0, sym_layout_.bytes));
    nseg_ = (c.H + 255) / 256;
    // KRB_RELAY=direct|rsag; default: direct all-pull for k <= 2, where it moves the
    // same NVLink bytes as reduce-scatter + all-gather with one sync instead of two
    relay_direct_ = k <= 2 ? 1 : 0;
    if (const char *e = std::getenv("KRB_RELAY")) {
      if (!std::strcmp(e, "direct")) relay_direct_ = 1;
      else if (!std::strcmp(e, "rsag")) relay_direct_ = 0;
      else throw std::runtime_error("KRB_RELAY must be direct or rsag");
    }
    if (relay_direct_ && k > 4) throw std::runtime_error("direct relay supports up to 4 ranks");
    // rsag phase order: the fixed pipeline rs(t+1) before ag(t) (measured ~2 % faster at
    // k = 4 than readiness order: every peer's all-gather waits on the reduce-scatters);
    // KRB_RELAY_ORDER=ready takes whichever phase is ready, in runs of ready tiles
    relay_ready_order_ = 0;
    if (const char *e = std::getenv("KRB_RELAY_ORDER")) {
      if (!std::strcmp(e, "ready")) relay_ready_order_ = 1;
      else if (!std::strcmp(e, "pipeline")) relay_ready_order_ = 0;
      else throw std::runtime_error("KRB_RELAY_ORDER must be ready or pipeline");
    }
    if (relay_ready_order_ && opts_.tiles > 32)
      throw std::runtime_error("KRB_RELAY_ORDER=ready supports up to 32 row tiles");
    if (const char *e = std::getenv("KRB_RELAY_TRACE"))
      if (std::atoi(e) > 0) {
        const size_t n = size_t(sm_count(opts_.device)) * kTraceSlots;
        trace_ = static_cast<unsigned long long *>(alloc(n * 8));
        KRB_CUDA(cudaMemset(trace_, 0, n * 8));
      }
    peers_.assign(k, nullptr);
    peers_[opts_.rank] = sym_;
  }
  KRB_CUDA(cudaStreamSynchronize(stream_));
}

Engine::~Engine() {
  cudaSetDevice(opts_.device);
  if (graph_) cudaGraphExecDestroy(graph_);
  for (void *p : allocs_) cudaFree(p);
  if (sym_) cudaFree(sym_);
  if (oflags_) cudaFree(oflags_);
  if (stream_) cudaStreamDestroy(stream_);
}

void Engine::set_peers(const std::vector<void *> &bases) {
  if (!mode_.split) return;
  if (int(bases.size()) != opts_.world) throw std::runtime_error("set_peers: wrong count");
  peers_ = bases;
  peers_[opts_.rank] = sym_;
}

// Bring tensor `name` (reference layout) into device staging memory.
void Engine::fetch(const std::string &name, __nv_bfloat16 *staging) {
  const TensorSpec &t = m_.at(name);
  const size_t n = t.numel();
  if (t.synth) {
    if (t.kind == "normal") {
      synth_normal_device(staging, n, synth_key(name.c_str(), t.seed), t.std_, t.mean, stream_);
    } else if (t.kind == "const") {
      fill_const_device(staging, n, float(t.value), stream_);
    } else if (t.kind == "transpose_of") {
      const TensorSpec &src = m_.at(t.alias);
      if (src.shape.size() != 2 || t.shape.size() != 2 || src.shape[0] != t.shape[1] ||
          src.shape[1] != t.shape[0])
        throw std::runtime_error("manifest: bad transpose_of for " + name);
      __nv_bfloat16 *tmp = static_cast<__nv_bfloat16 *>(nullptr);
      KRB_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&tmp), src.numel() * 2, stream_));
      fetch(t.alias, tmp);
      transpose_bf16(tmp, src.shape[1], staging, t.shape[1], int(src.shape[0]), int(src.shape[1]),
                     stream_);
      KRB_CUDA(cudaFreeAsync(tmp, stream_));
    } else {
      throw std::runtime_error("manifest: unknown synth kind " + t.kind);
    }
    return;
  }
  if (!weight_map_ || weight_map_dir_ != m_.dir) {
    const std::string path = m_.dir + "/weights.bin";
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("open weights.bin");
    struct stat st {};
    ::fstat(fd, &st);
    weight_map_bytes_ = size_t(st.st_size);
    weight_map_ = ::mmap(nullptr, weight_map_bytes_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (weight_map_ == MAP_FAILED) {
      weight_map_ = nullptr;
      throw std::runtime_error("mmap weights.bin");
    }
    weight_map_dir_ = m_.dir;
  }
  if (t.offset + t.bytes > weight_map_bytes_) throw std::runtime_error("weights.bin too short for " + name);
  KRB_CUDA(cudaMemcpyAsync(staging, static_cast<const char *>(weight_map_) + t.offset, t.bytes,
                           cudaMemcpyHostToDevice, stream_));
  KRB_CUDA(cudaStreamSynchronize(stream_));
}

void Engine::load_weights() {
  const ModelCfg &c = m_.cfg;
  const int H = c.H, D = c.D, r = opts_.rank;
  // largest tensor we stage
  size_t max_elems = 0;
  for (const auto &kv : m_.tensors) max_elems = std::max(max_elems, kv.second.numel());
  __nv_bfloat16 *stg = nullptr;
  KRB_CUDA(cudaMalloc(reinterpret_cast<void **>(&stg), max_elems * 2));
  auto A = [&](size_t elems) { return static_cast<__nv_bfloat16 *>(alloc(elems * 2)); };
  auto A16 = [&](size_t elems) { return static_cast<__half *>(alloc(elems * 2)); };
  auto as_bf = [](__half *p) { return reinterpret_cast<__nv_bfloat16 *>(p); };
  auto copy_into = [&](const std::string &name, __nv_bfloat16 *dst) {
    fetch(name, stg);
    KRB_CUDA(cudaMemcpyAsync(dst, stg, m_.at(name).numel() * 2, cudaMemcpyDeviceToDevice, stream_));
  };
  lw_.resize(c.L);
  const int nq = c.HQ * D, nkv = c.HKV * D;
  for (int l = 0; l < c.L; ++l) {
    const std::string p = layer_prefix(l);
    LayerW &w = lw_[l];
    if (l < layer_begin_ || l >= layer_end_) {
      // another pipeline stage's layer: only its input norm (the last layer of a
      // stage normalises with the next layer's ln1)
      w.ln1 = A(H);
      copy_into(p + "input_layernorm.weight", w.ln1);
      continue;
    }
    // fused QKV [nq + 2 nkv, H] K-major from q/k/v weight_t [H, n]
    // every GEMM weight is re-laid out in bf16, then converted to fp16 in place
    w.wqkv = A16(size_t(nqkv_) * H);
    const std::string roles[3] = {"q_proj", "k_proj", "v_proj"};
    const int widths[3] = {nq, nkv, nkv};
    int off = 0;
    for (int i = 0; i < 3; ++i) {
      fetch(p + roles[i] + ".weight_t", stg);
      transpose_bf16(stg, widths[i], as_bf(w.wqkv) + size_t(off) * H, H, H, widths[i], stream_);
      off += widths[i];
    }
    bf16_to_f16_inplace(w.wqkv, size_t(nqkv_) * H, stream_);
    if (c.bias) {
      w.bqkv = A(nqkv_);
      off = 0;
      for (int i = 0; i < 3; ++i) {
        copy_into(p + roles[i] + ".bias", w.bqkv + off);
        off += widths[i];
      }
    }
    // o_proj weight_t [nq, H] -> Wo [H, nq]
    w.wo = A16(size_t(H) * nq);
    fetch(p + "o_proj.weight_t", stg);
    transpose_bf16(stg, H, as_bf(w.wo), nq, nq, H, stream_);
    bf16_to_f16_inplace(w.wo, size_t(H) * nq, stream_);
    // gate/up weight_t [H, I]: this rank's column slab, interleaved per bn_gu_ block
    w.wgu = A16(size_t(gu_rows_) * H);
    KRB_CUDA(cudaMemsetAsync(w.wgu, 0, size_t(gu_rows_) * H * 2, stream_));
    const int half = bn_gu_ / 2;
    const int nblk = gu_rows_ / bn_gu_;
    for (int part = 0; part < 2; ++part) {
      fetch(p + (part == 0 ? "gate_proj.weight_t" : "up_proj.weight_t"), stg);
      for (int b = 0; b < nblk; ++b) {
        const int c0 = b * half;
        const int wdt = std::min(half, Iloc_ - c0);
        if (wdt <= 0) break;
        transpose_bf16(stg + size_t(r) * Iloc_ + c0, c.I,
                       as_bf(w.wgu) + (size_t(b) * bn_gu_ + part * half) * H, H, H, wdt, stream_);
      }
    }
    bf16_to_f16_inplace(w.wgu, size_t(gu_rows_) * H, stream_);
    // down weight_t [I, H]: rows [r*Iloc, (r+1)*Iloc) -> Wdown [H, Iloc]
    w.wdown = A16(size_t(H) * Iloc_);
    fetch(p + "down_proj.weight_t", stg);
    transpose_bf16(stg + size_t(r) * Iloc_ * H, H, as_bf(w.wdown), Iloc_, Iloc_, H, stream_);
    bf16_to_f16_inplace(w.wdown, size_t(H) * Iloc_, stream_);
    w.ln1 = A(H);
    copy_into(p + "input_layernorm.weight", w.ln1);
    w.ln2 = A(H);
    copy_into(p + "post_attention_layernorm.weight", w.ln2);
    if (c.qk_norm) {
      w.qn = A(D);
      copy_into(p + "q_norm.weight", w.qn);
      w.kn = A(D);
      copy_into(p + "k_norm.weight", w.kn);
    }
    KRB_CUDA(cudaStreamSynchronize(stream_));
  }
  embed_ = A(size_t(c.V) * H);
  copy_into("embed.weight", embed_);
  // only the logits engine (TP rank 0 of the last stage) keeps lm_head / final norm
  // (reference :1206-1208)
  if (has_logits()) {
    final_norm_ = A(H);
    copy_into("final_norm.weight", final_norm_);
    const TensorSpec &lm = m_.at("lm_head.weight_t");
    wlm_ = A16(size_t(c.V) * H);
    if (lm.synth && lm.kind == "transpose_of" && lm.alias == "embed.weight") {
      // tied: lm_head.weight_t == embed^T, i.e. Wlm [V,H] == embed (an fp16 copy; the
      // gather keeps reading the bf16 table)
      KRB_CUDA(cudaMemcpyAsync(wlm_, embed_, size_t(c.V) * H * 2, cudaMemcpyDeviceToDevice,
                               stream_));
    } else {
      fetch("lm_head.weight_t", stg);
      transpose_bf16(stg, c.V, as_bf(wlm_), H, H, c.V, stream_);
    }
    bf16_to_f16_inplace(wlm_, size_t(c.V) * H, stream_);
  }
  // rope tables [1,1,max_pos,D] -> used as [max_pos, D]
  cos_ = A(size_t(c.max_pos) * D);
  copy_into("rope.cos", cos_);
  sin_ = A(size_t(c.max_pos) * D);
  copy_into("rope.sin", sin_);
  KRB_CUDA(cudaStreamSynchronize(stream_));
  KRB_CUDA(cudaFree(stg));
  if (weight_map_) {
    ::munmap(weight_map_, weight_map_bytes_);
    weight_map_ = nullptr;
    weight_map_dir_.clear();
  }
}

void Engine::alloc_activations() {
  const ModelCfg &c = m_.cfg;
  const size_t S = size_t(opts_.seq), H = size_t(c.H);
  auto A = [&](size_t elems) { return static_cast<__half *>(alloc(elems * 2)); };
  auto F = [&](size_t elems) { return static_cast<float *>(alloc(elems * 4)); };
  h0_ = F(S * H);
  h1_ = F(S * H);
  x_ = A(S * H);
  qkv_ = A(S * size_t(nqkv_));
  attn_ = A(S * size_t(c.HQ) * c.D);
  o_ = A(S * H);
  act_ = A(S * size_t(Iloc_));
  down_ = A(S * H);
  if (mode_.tp && mode_.world > 1 && !mode_.split) red_ = A(S * H);
  hf_ = F(S * H);
  delta_ = F(S * H);
  xf_ = A(S * H);
  if (has_logits()) logits_ = A(size_t(lm_rows_) * size_t(c.V));
  last_f32_ = static_cast<float *>(alloc(size_t(c.V) * 4));
  // tcgen05 attention reads V transposed ([kv head * D + d][key])
  if (c.D != 64 && c.D != 128) throw std::runtime_error("attention: head_dim must be 64 or 128");
  ldvt_ = (long(S) + 7) / 8 * 8;
  vt_ = reinterpret_cast<__half *>(A(size_t(c.HKV) * c.D * ldvt_));
  // token ids (ids.bin int64 [S], reference UploadIds :473-485)
  ids_ = static_cast<int64_t *>(alloc(S * 8));
  std::ifstream f(m_.dir + "/ids.bin", std::ios::binary | std::ios::ate);
  if (!f) throw std::runtime_error("ids.bin");
  const size_t bytes = size_t(f.tellg());
  if (bytes != S * 8) throw std::runtime_error("ids size != seq");
  f.seekg(0);
  std::vector<int64_t> ids(S);
  f.read(reinterpret_cast<char *>(ids.data()), std::streamsize(bytes));
  KRB_CUDA(cudaMemcpy(ids_, ids.data(), bytes, cudaMemcpyHostToDevice));
}

// ---- stage timing helper
namespace {
struct StageRec {
  cudaStream_t s;
  StageTimes *st;
  std::vector<std::pair<double *, std::pair<cudaEvent_t, cudaEvent_t>>> *events;
  cudaEvent_t a = nullptr;
  double *slot = nullptr;
  StageRec(cudaStream_t s_, StageTimes *st_,
           std::vector<std::pair<double *, std::pair<cudaEvent_t, cudaEvent_t>>> *ev)
      : s(s_), st(st_), events(ev) {}
  void begin(double *slot_) {
    if (!st) return;
    slot = slot_;
    KRB_CUDA(cudaEventCreate(&a));
    KRB_CUDA(cudaEventRecord(a, s));
  }
  void end() {
    if (!st) return;
    cudaEvent_t b;
    KRB_CUDA(cudaEventCreate(&b));
    KRB_CUDA(cudaEventRecord(b, s));
    events->push_back({slot, {a, b}});
  }
};
thread_local std::vector<std::pair<double *, std::pair<cudaEvent_t, cudaEvent_t>>> *g_events =
    nullptr;
}  // namespace

void Engine::prologue(StageTimes *st) {
  const ModelCfg &c = m_.cfg;
  StageRec rec(stream_, st, g_events);
  if (mode_.split) {
    bump_epoch(reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(sym_) + sym_layout_.epoch()), stream_);
    ++launches_;
  }
  if (fuse_oproj_) {
    bump_epoch(reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(oflags_) + oflags_layout_.epoch()),
               stream_);
    ++launches_;
  }
  rec.begin(st ? &st->embed : nullptr);
  embed_f32(ids_, embed_, h0_, opts_.seq, c.H, c.V, status_, stream_);
  add_rmsnorm_res_f32(h0_, static_cast<const float *>(nullptr), lw_[0].ln1, x_, nullptr, opts_.seq,
                      c.H, float(c.eps), stream_);
  launches_ += 2;
  rec.end();
}

// Add + RMSNorm on the fp32 residual stream: one fused kernel, or (unfused serial
// modes, qwen_main.cpp:976-979) an add pass followed by a separate RMSNorm pass.
void Engine::add_norm(const float *res, const __half *delta, const __nv_bfloat16 *gamma,
                      __half *y, float *sum) {
  const ModelCfg &c = m_.cfg;
  const float eps = float(c.eps);
  add_rmsnorm_res_f32(res, delta, gamma, y, sum, opts_.seq, c.H, eps, stream_);
  launches_ += 1;
  if (!mode_.fused) {
    add_rmsnorm_res_f32(sum, static_cast<const float *>(nullptr), gamma, y, nullptr, opts_.seq, c.H,
                        eps, stream_);
    launches_ += 1;
  }
}

void Engine::layer(int l, StageTimes *st) {
  const ModelCfg &c = m_.cfg;
  const int S = opts_.seq, H = c.H, D = c.D;
  const float eps = float(c.eps);
  const LayerW &w = lw_[l];
  StageRec rec(stream_, st, g_events);
  launches_ += 4;  // QKV GEMM, attention, o_proj GEMM, gate/up GEMM (others where they launch)
  rec.begin(st ? &st->qkv : nullptr);
  if (fuse_rope_) {
    // QK-norm and RoPE in the QKV GEMM's epilogue (no separate pass over q / k)
    // (and writes the fp16 V^T the attention reads: no separate transpose)
    gemm_qkv_rope<__half>(x_, H, w.wqkv, H, qkv_, nqkv_, c.bias ? w.bqkv : nullptr, S, H, c.HQ,
                          c.HKV, D, cos_, sin_, c.qk_norm ? w.qn : nullptr,
                          c.qk_norm ? w.kn : nullptr, eps, status_, stream_, vt_, ldvt_);
    rec.end();
  } else {
    // unfused serial modes: the reference's separate ops (qwen_main.cpp:1336-1357, 567-582)
    gemm_store<__half>(x_, H, w.wqkv, H, qkv_, nqkv_, c.bias ? w.bqkv : nullptr, S, nqkv_, H, 0,
                       0, status_, stream_);
    rec.end();
    rec.begin(st ? &st->rope : nullptr);
    qk_norm_rope<__half>(qkv_, S, c.HQ, c.HKV, D, cos_, sin_, c.qk_norm ? w.qn : nullptr,
                         c.qk_norm ? w.kn : nullptr, eps, stream_);
    ++launches_;
    rec.end();
  }
  rec.begin(st ? &st->attn : nullptr);
  if (!fuse_rope_) {
    attention_vt<__half>(qkv_, vt_, ldvt_, S, c.HQ, c.HKV, D, stream_);  // else the QKV epilogue writes it
    ++launches_;
  }
  attention_tc<__half>(qkv_, vt_, ldvt_, attn_, S, c.HQ, c.HKV, D,
                       float(1.0 / std::sqrt(double(D))), status_, stream_);
  rec.end();
  if (fuse_oproj_) {
    // o_proj, residual add and ln2 in one kernel: the relay kernel at k = 1 (the fp32
    // o_proj rows land in h1, its relay warps add the residual and normalise each row tile
    // as soon as its GEMM tiles are done, while the GEMM continues on the next tiles)
    RelayArgs ra{};
    ra.S = S;
    ra.H = H;
    ra.K = c.HQ * D;
    ra.T = o_tiles_;
    ra.k = 1;
    ra.rank = 0;
    ra.R = S / o_tiles_;
    ra.Rk = ra.R;
    ra.nseg = (H + 255) / 256;
    ra.peer_base[0] = static_cast<uint8_t *>(oflags_);
    ra.local_base = static_cast<uint8_t *>(oflags_);
    ra.flag_off = oflags_layout_.flag_off;
    ra.epoch = reinterpret_cast<const uint32_t *>(static_cast<uint8_t *>(oflags_) +
                                                  oflags_layout_.epoch());
    ra.layer = l;
    ra.L = c.L;
    ra.resid = h0_;
    ra.gamma = w.ln2;
    ra.sum_out = h1_;
    ra.x_out = reinterpret_cast<__nv_bfloat16 *>(x_);  // holds fp16 (the relay's T)
    ra.eps = eps;
    ra.do_norm = 1;
    ra.timeout_ns = flag_timeout_ns_;
    ra.status = status_;
    rec.begin(st ? &st->o : nullptr);
    relay_down_layer(attn_, c.HQ * D, w.wo, c.HQ * D, bn_down_, ra, stream_);  // counted above
    rec.end();
  } else if (mode_.fused) {
    // o_proj output kept in fp32 (no bf16 rounding of o); residual add fused into the norm
    rec.begin(st ? &st->o : nullptr);
    gemm_f32out(attn_, c.HQ * D, w.wo, c.HQ * D, delta_, H, S, H, c.HQ * D, 0, status_, stream_);
    rec.end();
    rec.begin(st ? &st->addnorm : nullptr);
    add_rmsnorm_res_f32(h0_, delta_, w.ln2, x_, h1_, S, H, eps, stream_);
    ++launches_;
    rec.end();
  } else {
    rec.begin(st ? &st->o : nullptr);
    gemm_store<__half>(attn_, c.HQ * D, w.wo, c.HQ * D, o_, H, nullptr, S, H, c.HQ * D, 0, 0,
                       status_, stream_);
    rec.end();
    rec.begin(st ? &st->addnorm : nullptr);
    add_norm(h0_, o_, w.ln2, x_, h1_);
    rec.end();
  }
  rec.begin(st ? &st->gateup : nullptr);
  gemm_silu<__half>(x_, H, w.wgu, H, act_, Iloc_, S, Iloc_, H, bn_gu_, 0, status_, stream_);
  rec.end();

  const bool last = (l + 1 == c.L);
  const __nv_bfloat16 *gamma = last ? final_norm_ : lw_[l + 1].ln1;
  float *sum_out = last ? hf_ : h0_;
  __half *x_out = last ? xf_ : x_;
  const bool do_norm = !last || opts_.rank == 0;
  down_stage(l, st, gamma ? gamma : lw_[l].ln1, sum_out, x_out, do_norm);  // rank != 0, last: unused
}

void Engine::down_stage(int l, StageTimes *st, const __nv_bfloat16 *gamma, float *sum_out,
                        __half *x_out, bool do_norm) {
  const ModelCfg &c = m_.cfg;
  const int S = opts_.seq, H = c.H;
  const float eps = float(c.eps);
  const LayerW &w = lw_[l];
  StageRec rec(stream_, st, g_events);
  if (mode_.split) {
    RelayArgs ra{};
    ra.S = S;
    ra.H = H;
    ra.K = Iloc_;
    ra.T = opts_.tiles;
    ra.k = opts_.world;
    ra.rank = opts_.rank;
    ra.R = S / opts_.tiles;
    ra.Rk = ra.R / ra.k;
    ra.nseg = nseg_;
    for (int i = 0; i < ra.k; ++i) {
      if (!peers_[i]) throw std::runtime_error("relay: peer mapping missing");
      ra.peer_base[i] = static_cast<uint8_t *>(peers_[i]);
    }
    ra.local_base = static_cast<uint8_t *>(sym_);
    ra.part_off = sym_layout_.part_off;
    ra.red_off = sym_layout_.red_off;
    ra.flag_off = sym_layout_.flag_off;
    ra.direct = relay_direct_;
    ra.ready_order = relay_ready_order_;
    ra.epoch = reinterpret_cast<const uint32_t *>(static_cast<uint8_t *>(sym_) + sym_layout_.epoch());
    ra.layer = l;
    ra.L = c.L;
    ra.resid = h1_;
    ra.gamma = gamma;
    ra.sum_out = sum_out;
    ra.x_out = reinterpret_cast<__nv_bfloat16 *>(x_out);  // holds fp16 (the relay's T)
    ra.eps = eps;
    ra.do_norm = do_norm ? 1 : 0;
    ra.timeout_ns = flag_timeout_ns_;
    ra.status = status_;
    ra.trace = trace_;
    rec.begin(st ? &st->relay : nullptr);
    relay_down_layer(act_, Iloc_, w.wdown, Iloc_, bn_down_, ra, stream_);
    ++launches_;
    rec.end();
    return;
  }
  ++launches_;
  if (mode_.fused && opts_.world == 1) {
    // single device: down output kept in fp32, residual add fused into the norm
    rec.begin(st ? &st->down : nullptr);
    gemm_f32out(act_, Iloc_, w.wdown, Iloc_, delta_, H, S, H, Iloc_, bn_down_, status_, stream_);
    rec.end();
    rec.begin(st ? &st->addnorm2 : nullptr);
    add_rmsnorm_res_f32(h1_, delta_, gamma, x_out, sum_out, S, H, eps, stream_);
    ++launches_;
    rec.end();
    return;
  }
  rec.begin(st ? &st->down : nullptr);
  gemm_store<__half>(act_, Iloc_, w.wdown, Iloc_, down_, H, nullptr, S, H, Iloc_, bn_down_, 0,
                     status_, stream_);
  rec.end();
  const __half *red = down_;
  if (mode_.tp && mode_.world > 1) {
    if (!nccl_) throw std::runtime_error("tp: NCCL communicator missing");
    rec.begin(st ? &st->allreduce : nullptr);
    if (ncclAllReduce(down_, red_, size_t(S) * H, ncclHalf, ncclSum, nccl_, stream_) != ncclSuccess)
      throw std::runtime_error("ncclAllReduce failed");
    rec.end();
    red = red_;
  }
  if (do_norm) {
    rec.begin(st ? &st->addnorm2 : nullptr);
    add_norm(h1_, red, gamma, x_out, sum_out);
    rec.end();
  }
}

void Engine::epilogue(StageTimes *st) {
  if (!has_logits()) return;
  const ModelCfg &c = m_.cfg;
  StageRec rec(stream_, st, g_events);
  ++launches_;
  rec.begin(st ? &st->lm_head : nullptr);
  const int r0 = opts_.seq - lm_rows_;
  gemm_store<__half>(xf_ + size_t(r0) * c.H, c.H, wlm_, c.H, logits_, c.V, nullptr, lm_rows_, c.V,
                     c.H, 0, 0, status_, stream_);
  rec.end();
}

void Engine::enqueue() { enqueue_stage(nullptr); }

void Engine::microdag_enqueue(StageTimes *st) {
  if (mode_.split) {
    bump_epoch(reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(sym_) + sym_layout_.epoch()), stream_);
    ++launches_;
  }
  down_stage(0, st, md_gamma_, hf_, xf_, true);  // every rank normalises its rows
}

// Micro-DAG inputs, generated on the device: X_r, W_r with seed
// md_seed + rank, R with md_seed, gamma = 1.
void Engine::load_microdag() {
  const ModelCfg &c = m_.cfg;
  const size_t S = size_t(opts_.seq), H = size_t(c.H), K = size_t(Iloc_);
  const uint64_t sr = opts_.md_seed + uint64_t(opts_.rank);
  auto A = [&](size_t elems) { return static_cast<__nv_bfloat16 *>(alloc(elems * 2)); };
  auto A16 = [&](size_t elems) { return static_cast<__half *>(alloc(elems * 2)); };
  auto F = [&](size_t elems) { return static_cast<float *>(alloc(elems * 4)); };
  __nv_bfloat16 *stg = nullptr;
  KRB_CUDA(cudaMalloc(reinterpret_cast<void **>(&stg), std::max(K * H, S * H) * 2));
  lw_.resize(1);
  // W_r [K, H] (the reference's down_proj.weight_t layout) -> Wdown [H, K]
  // bf16 values (the configuration's dtype), held in fp16 exactly like the engine's weights
  lw_[0].wdown = A16(H * K);
  synth_normal_device(stg, K * H, synth_key("microdag.W_down", sr), 0.02, 0.0, stream_);
  transpose_bf16(stg, H, reinterpret_cast<__nv_bfloat16 *>(lw_[0].wdown), K, K, H, stream_);
  bf16_to_f16_inplace(lw_[0].wdown, H * K, stream_);
  act_ = A16(S * K);
  synth_normal_device(reinterpret_cast<__nv_bfloat16 *>(act_), S * K, synth_key("microdag.X", sr),
                      1.0, 0.0, stream_);
  bf16_to_f16_inplace(act_, S * K, stream_);
  h1_ = F(S * H);  // residual R, exact in fp32
  synth_normal_device(stg, S * H, synth_key("microdag.R", opts_.md_seed), 1.0, 0.0, stream_);
  bf16_row_to_f32(stg, h1_, int(S * H), stream_);
  md_gamma_ = A(H);
  fill_const_device(md_gamma_, H, 1.0f, stream_);
  hf_ = F(S * H);
  xf_ = A16(S * H);
  delta_ = F(S * H);
  down_ = A16(S * H);
  if (mode_.world > 1 && !mode_.split) red_ = A16(S * H);
  KRB_CUDA(cudaStreamSynchronize(stream_));
  KRB_CUDA(cudaFree(stg));
}

void Engine::enqueue_stage(const float *h_in) {
  KRB_CUDA(cudaSetDevice(opts_.device));
  launches_ = 0;
  if (opts_.microdag) {
    microdag_enqueue(nullptr);
    return;
  }
  const size_t SH = size_t(opts_.seq) * m_.cfg.H;
  if (layer_begin_ == 0) {
    prologue(nullptr);
  } else {
    // later pipeline stage: the previous stage's residual stream, then this stage's
    // first input norm (qwen_main.cpp:1459-1465)
    if (!h_in) throw std::runtime_error("pp: stage input missing");
    KRB_CUDA(cudaMemcpyAsync(h0_, h_in, SH * 4, cudaMemcpyDeviceToDevice, stream_));
    add_rmsnorm_res_f32(h0_, static_cast<const float *>(nullptr), lw_[layer_begin_].ln1, x_,
                        nullptr, opts_.seq, m_.cfg.H, float(m_.cfg.eps), stream_);
    launches_ += 1;
  }
  for (int l = layer_begin_; l < layer_end_; ++l) {
    layer(l, nullptr);
    if (dump_) {
      const bool last = (l + 1 == m_.cfg.L);
      if (!last || opts_.rank == 0)
        KRB_CUDA(cudaMemcpyAsync(dump_ + size_t(l) * SH, last ? hf_ : h0_, SH * 4,
                                 cudaMemcpyDeviceToDevice, stream_));
    }
  }
  epilogue(nullptr);
}

void Engine::set_layer_dump(bool on) {
  KRB_CUDA(cudaSetDevice(opts_.device));
  if (on && !dump_) {
    dump_ = static_cast<float *>(alloc(size_t(m_.cfg.L) * opts_.seq * m_.cfg.H * 4));
  } else if (!on) {
    dump_ = nullptr;  // memory stays in allocs_ until destruction
  }
}

std::vector<float> Engine::layer_hidden(int l) {
  if (!dump_) throw std::runtime_error("layer dumps are off");
  if (l < 0 || l >= m_.cfg.L) throw std::runtime_error("layer out of range");
  const size_t SH = size_t(opts_.seq) * m_.cfg.H;
  std::vector<float> out(SH);
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaStreamSynchronize(stream_));
  KRB_CUDA(cudaMemcpy(out.data(), dump_ + size_t(l) * SH, SH * 4, cudaMemcpyDeviceToHost));
  return out;
}

void Engine::enqueue_host(const int64_t *ids_host, float *last_logits_host) {
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaMemcpyAsync(ids_, ids_host, size_t(opts_.seq) * 8, cudaMemcpyHostToDevice, stream_));
  run();
  if (has_logits() && last_logits_host) {
    const ModelCfg &c = m_.cfg;
    f16_to_f32(logits_ + size_t(lm_rows_ - 1) * c.V, last_f32_, c.V, stream_);
    KRB_CUDA(cudaMemcpyAsync(last_logits_host, last_f32_, size_t(c.V) * 4, cudaMemcpyDeviceToHost,
                             stream_));
  }
}

void Engine::capture_graph() {
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaStreamSynchronize(stream_));
  cudaGraph_t g = nullptr;
  KRB_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
  try {
    enqueue();
  } catch (...) {
    cudaStreamEndCapture(stream_, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  KRB_CUDA(cudaStreamEndCapture(stream_, &g));
  if (graph_) cudaGraphExecDestroy(graph_);
  KRB_CUDA(cudaGraphInstantiate(&graph_, g, 0));
  cudaGraphDestroy(g);
}

void Engine::run() {
  if (graph_) {
    KRB_CUDA(cudaSetDevice(opts_.device));
    KRB_CUDA(cudaGraphLaunch(graph_, stream_));
  } else {
    enqueue();
  }
}

void Engine::sync() {
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaStreamSynchronize(stream_));
}

uint32_t Engine::read_status() {
  uint32_t v = 0;
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaMemcpy(&v, status_, 4, cudaMemcpyDeviceToHost));
  return v;
}

StageTimes Engine::instrumented_run() {
  if (mode_.pp) throw std::runtime_error("stage times are not available in pp modes");
  KRB_CUDA(cudaSetDevice(opts_.device));
  std::vector<std::pair<double *, std::pair<cudaEvent_t, cudaEvent_t>>> events;
  g_events = &events;
  StageTimes st;
  cudaEvent_t a, b;
  KRB_CUDA(cudaEventCreate(&a));
  KRB_CUDA(cudaEventCreate(&b));
  KRB_CUDA(cudaEventRecord(a, stream_));
  launches_ = 0;
  try {
    if (opts_.microdag) {
      microdag_enqueue(&st);
    } else {
      prologue(&st);
      for (int l = 0; l < m_.cfg.L; ++l) layer(l, &st);
      epilogue(&st);
    }
  } catch (...) {
    g_events = nullptr;
    throw;
  }
  g_events = nullptr;
  KRB_CUDA(cudaEventRecord(b, stream_));
  KRB_CUDA(cudaStreamSynchronize(stream_));
  float ms = 0;
  KRB_CUDA(cudaEventElapsedTime(&ms, a, b));
  st.total = ms * 1000.0;
  for (auto &e : events) {
    KRB_CUDA(cudaEventElapsedTime(&ms, e.second.first, e.second.second));
    *e.first += ms * 1000.0;
    cudaEventDestroy(e.second.first);
    cudaEventDestroy(e.second.second);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return st;
}

std::vector<float> Engine::last_logits() {
  const ModelCfg &c = m_.cfg;
  std::vector<float> out;
  if (!has_logits()) return out;
  KRB_CUDA(cudaSetDevice(opts_.device));
  f16_to_f32(logits_ + size_t(lm_rows_ - 1) * c.V, last_f32_, c.V, stream_);
  out.resize(c.V);
  KRB_CUDA(cudaMemcpyAsync(out.data(), last_f32_, size_t(c.V) * 4, cudaMemcpyDeviceToHost, stream_));
  KRB_CUDA(cudaStreamSynchronize(stream_));
  return out;
}

const float *Engine::hidden_ptr() const { return hf_; }

std::vector<unsigned long long> Engine::relay_trace() {
  std::vector<unsigned long long> out;
  if (!trace_) return out;
  const size_t n = size_t(sm_count(opts_.device)) * kTraceSlots;
  out.resize(n);
  KRB_CUDA(cudaSetDevice(opts_.device));
  KRB_CUDA(cudaStreamSynchronize(stream_));
  KRB_CUDA(cudaMemcpy(out.data(), trace_, n * 8, cudaMemcpyDeviceToHost));
  return out;
}

Engine::Verdict Engine::verify() {
  Verdict v;
  if (!has_logits()) return v;
  const std::vector<float> got = last_logits();
  const int V = m_.cfg.V;
  float best = -INFINITY;
  double sum = 0;
  for (int i = 0; i < V; ++i) {
    if (got[i] > best) {
      best = got[i];
      v.argmax = i;
    }
    sum += std::fabs(double(got[i]));
  }
  v.abs_mean = sum / V;
  std::ifstream rf(m_.dir + "/ref_last_logits.bin", std::ios::binary);
  if (rf) {
    std::vector<float> ref(V);
    rf.read(reinterpret_cast<char *>(ref.data()), std::streamsize(size_t(V) * 4));
    if (rf.gcount() == std::streamsize(size_t(V) * 4)) {
      v.has_ref = true;
      for (int i = 0; i < V; ++i) v.maxdiff = std::max(v.maxdiff, std::fabs(double(got[i]) - ref[i]));
    }
  }
  try {
    json::Value rj = json::parse_file(m_.dir + "/ref.json");
    v.ref_argmax = int(rj.number_or("argmax_last", -1));
  } catch (...) {
  }
  return v;
}

}  // namespace krb
