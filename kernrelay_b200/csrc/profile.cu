// kr_qwen_profile_many: the planner's per-op k-granularity cost table, measured
// on B200 with the production kernels (reference Qwen::ProfileMany,
// qwen_main.cpp:1535-1783).  For each case {op, k} the op is split into k row
// slices (k head groups for attention), the k launches are captured in one CUDA
// graph, replayed 20 times between two events, three times; best/median of the
// per-replay device time are reported with the reference's field names.
//
// Ops fused away on B200 (add into add_rmsnorm, silu and mul into the gate/up
// GEMM epilogue, matmul_up into matmul_gate) are reported with best_us 0 and a
// "fused_into" field, so a planner does not double count them.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <sstream>

#include "json_min.hpp"
#include "kernrelay.h"
#include "model.h"

namespace krb {

std::string Engine::profile_many(const std::string &spec_path) {
  json::Value spec = json::parse_file(spec_path);
  const ModelCfg &c = m_.cfg;
  const int S = opts_.seq, H = c.H, D = c.D;
  const int nq = c.HQ * D, nkv = c.HKV * D;
  const float eps = float(c.eps);
  const LayerW &w = lw_[0];
  KRB_CUDA(cudaSetDevice(opts_.device));
  std::vector<std::string> cases;
  for (const auto &cs : spec.at("cases").arr) {
    const std::string op = cs.string_or("op", "");
    const int k = int(cs.number_or("k", 1));
    if (k < 1 || S % k) continue;
    const int per = S / k;
    std::function<void(int)> call;  // enqueue slice i
    std::string shape, fused;
    auto mm = [&](const __half *A, int lda, const __half *B, __half *C, int ldc, int N, int K) {
      shape = "matmul|" + std::to_string(S) + "x" + std::to_string(K) + "x" + std::to_string(N);
      call = [=](int i) {
        gemm_store<__half>(A + size_t(i) * per * lda, lda, B, K, C + size_t(i) * per * ldc, ldc,
                           nullptr, per, N, K, 0, 0, status_, stream_);
      };
    };
    if (op == "matmul_q") {
      mm(x_, H, w.wqkv, qkv_, nqkv_, nq, H);
    } else if (op == "matmul_k") {
      mm(x_, H, w.wqkv + size_t(nq) * H, qkv_ + nq, nqkv_, nkv, H);
    } else if (op == "matmul_v") {
      mm(x_, H, w.wqkv + size_t(nq + nkv) * H, qkv_ + nq + nkv, nqkv_, nkv, H);
    } else if (op == "matmul_o") {
      mm(attn_, nq, w.wo, o_, H, H, nq);
    } else if (op == "matmul_down") {
      mm(act_, Iloc_, w.wdown, down_, H, H, Iloc_);
    } else if (op == "matmul_lm") {
      if (opts_.rank != 0 || lm_rows_ != S) continue;
      mm(xf_, H, wlm_, logits_, c.V, c.V, H);
    } else if (op == "matmul_gate") {
      shape = "matmul_silu|" + std::to_string(S) + "x" + std::to_string(H) + "x" +
              std::to_string(2 * Iloc_);
      call = [=](int i) {
        gemm_silu<__half>(x_ + size_t(i) * per * H, H, w.wgu, H, act_ + size_t(i) * per * Iloc_,
                          Iloc_, per, Iloc_, H, bn_gu_, 0, status_, stream_);
      };
    } else if (op == "matmul_up" || op == "silu" || op == "mul") {
      fused = "matmul_gate";
    } else if (op == "add") {
      fused = "add_rmsnorm";
    } else if (op == "rmsnorm") {
      shape = "rmsnorm|" + std::to_string(S) + "x" + std::to_string(H);
      call = [=](int i) {
        rmsnorm_act<__half>(x_ + size_t(i) * per * H, w.ln1, o_ + size_t(i) * per * H, per, H, eps,
                            stream_);
      };
    } else if (op == "add_rmsnorm") {
      shape = "add_rmsnorm|" + std::to_string(S) + "x" + std::to_string(H);
      call = [=](int i) {
        const size_t off = size_t(i) * per * H;
        add_rmsnorm_res_f32(h0_ + off, o_ + off, w.ln2, x_ + off, h1_ + off, per, H, eps, stream_);
      };
    } else if (op == "rope") {
      shape = "rope|" + std::to_string(S) + "x" + std::to_string(nq + nkv);
      call = [=](int i) {
        qk_norm_rope<__half>(qkv_ + size_t(i) * per * nqkv_, per, c.HQ, c.HKV, D,
                             cos_ + size_t(i) * per * D, sin_ + size_t(i) * per * D,
                             c.qk_norm ? w.qn : nullptr, c.qk_norm ? w.kn : nullptr, eps, stream_);
      };
    } else if (op == "embedding") {
      shape = "embedding|" + std::to_string(S) + "x" + std::to_string(H);
      call = [=](int i) {
        embed_f32(ids_ + size_t(i) * per, embed_, h0_ + size_t(i) * per * H, per, H, c.V, status_,
                  stream_);
      };
    } else if (op == "attention") {
      if (c.HQ % k) continue;
      const int hq = c.HQ / k;
      const bool kv_div = c.HKV % k == 0;
      const int hkv = kv_div ? c.HKV / k : 1;
      shape = "attention|" + std::to_string(c.HQ) + "x" + std::to_string(S) + "x" + std::to_string(D);
      // k head groups; with k > HKV each group gets one KV head, cycling (reference :1689-1704)
      // each group: V^T of its KV heads, then the tcgen05 attention over its query heads
      // (the same two kernels as the prefill's attention stage)
      call = [=](int g) {
        const int kv_off = kv_div ? g * hkv : g % c.HKV;
        const int group = std::max(1, hq / hkv);
        attention_vt<__half>(qkv_, vt_, ldvt_, S, c.HQ, c.HKV, D, stream_, kv_off, hkv);
        attention_tc<__half>(qkv_, vt_, ldvt_, attn_, S, c.HQ, c.HKV, D,
                             float(1.0 / std::sqrt(double(D))), status_, stream_, g * hq, hq,
                             kv_off, group);
      };
    } else {
      continue;
    }
    std::ostringstream os;
    if (!fused.empty()) {
      os << "{\"op\":\"" << op << "\",\"k\":" << k << ",\"rows\":" << S << ",\"best_us\":0"
         << ",\"median_us\":0,\"per_tile_us\":0,\"fused_into\":\"" << fused << "\",\"graph\":true}";
      cases.push_back(os.str());
      continue;
    }
    try {
      cudaGraph_t g = nullptr;
      cudaGraphExec_t ge = nullptr;
      KRB_CUDA(cudaStreamSynchronize(stream_));
      KRB_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
      try {
        for (int i = 0; i < k; ++i) call(i);
      } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      KRB_CUDA(cudaStreamEndCapture(stream_, &g));
      KRB_CUDA(cudaGraphInstantiate(&ge, g, 0));
      cudaGraphDestroy(g);
      const int repeats = 20;
      for (int wu = 0; wu < 2; ++wu) KRB_CUDA(cudaGraphLaunch(ge, stream_));
      KRB_CUDA(cudaStreamSynchronize(stream_));
      cudaEvent_t e0, e1;
      KRB_CUDA(cudaEventCreate(&e0));
      KRB_CUDA(cudaEventCreate(&e1));
      std::vector<double> dev;
      for (int it = 0; it < 3; ++it) {
        KRB_CUDA(cudaEventRecord(e0, stream_));
        for (int r = 0; r < repeats; ++r) KRB_CUDA(cudaGraphLaunch(ge, stream_));
        KRB_CUDA(cudaEventRecord(e1, stream_));
        KRB_CUDA(cudaEventSynchronize(e1));
        float ms = 0;
        KRB_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        dev.push_back(double(ms) * 1000.0 / repeats);
      }
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      cudaGraphExecDestroy(ge);
      std::vector<double> sorted = dev;
      std::sort(sorted.begin(), sorted.end());
      os << "{\"op\":\"" << op << "\",\"k\":" << k << ",\"rows\":" << S << ",\"shape\":\"" << shape
         << "\",\"best_us\":" << sorted.front() << ",\"median_us\":" << sorted[sorted.size() / 2]
         << ",\"per_tile_us\":" << sorted.front() / k << ",\"graph\":true,\"samples_us\":[";
      for (size_t i = 0; i < dev.size(); ++i) os << (i ? "," : "") << dev[i];
      os << "]}";
    } catch (const std::exception &ex) {
      os.str("");
      os << "{\"op\":\"" << op << "\",\"k\":" << k << ",\"error\":\"" << json::escape(ex.what())
         << "\"}";
    }
    cases.push_back(os.str());
  }
  const uint32_t st = read_status();
  if (st) throw std::runtime_error("device status " + std::to_string(st) + " during profiling");
  std::ostringstream out;
  out << "{\"model\":\"" << json::escape(m_.dir) << "\",\"device\":\"B200\",\"cases\":[";
  for (size_t i = 0; i < cases.size(); ++i) out << (i ? "," : "") << cases[i];
  out << "]}";
  return out.str();
}

}  // namespace krb

extern "C" __attribute__((visibility("default"))) int kr_qwen_profile_many(
    const char *model_dir, const char *spec_json, int seq, int device, char *out, size_t out_cap) {
  try {
    if (!model_dir || !*model_dir) throw std::runtime_error("model path required");
    if (!spec_json) throw std::runtime_error("spec path required");
    krb::EngineOpts o;
    o.model_dir = model_dir;
    o.mode = "serial";
    o.seq = seq;
    o.device = device;
    krb::Engine e(o);
    e.run();
    e.sync();
    const std::string res = e.profile_many(spec_json);
    if (!out || out_cap < res.size() + 1) throw std::runtime_error("output buffer too small");
    std::memcpy(out, res.c_str(), res.size() + 1);
    return 0;
  } catch (const std::exception &ex) {
    if (out && out_cap) {
      const std::string msg = std::string("{\"error\":\"") + krb::json::escape(ex.what()) + "\"}";
      std::snprintf(out, out_cap, "%s", msg.c_str());
    }
    return 1;
  }
}
