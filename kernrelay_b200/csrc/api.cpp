// C ABI of libkernrelay.so: the reference's six entry points (kernrelay.h) and
// the B200 extensions (kernrelay_b200.h).  No C++ exception crosses the ABI.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <barrier>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "json_min.hpp"
#include "kernrelay.h"
#include "kernrelay_b200.h"
#include "model.h"
#include "plan.h"
#include "ptx.cuh"
#include "synth.cuh"

#define KRB_EXPORT extern "C" __attribute__((visibility("default")))

using Clock = std::chrono::steady_clock;

namespace {

thread_local std::string g_last_error;

double us_between(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double, std::micro>(b - a).count();
}

int fail(const std::exception &e) {
  g_last_error = e.what();
  return 1;
}

int write_out(const std::string &res, char *out, size_t cap) {
  if (!out || cap < res.size() + 1) throw std::runtime_error("output buffer too small");
  std::memcpy(out, res.c_str(), res.size() + 1);
  return 0;
}

int write_error(const std::string &what, char *out, size_t cap) {
  g_last_error = what;
  if (out && cap) {
    const std::string msg = "{\"error\":\"" + krb::json::escape(what) + "\"}";
    std::snprintf(out, cap, "%s", msg.c_str());
  }
  return 1;
}

cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

std::string fmt(double v) {
  char b[64];
  std::snprintf(b, sizeof(b), "%.3f", v);
  return b;
}

void stats(const std::vector<double> &s, double *best, double *typ) {
  std::vector<double> v = s;
  std::sort(v.begin(), v.end());
  *best = v.empty() ? 0 : v.front();
  *typ = v.empty() ? 0 : v[v.size() / 2];
}

std::string samples_json(const std::vector<double> &s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) {
    if (i) o += ",";
    o += fmt(s[i]);
  }
  return o + "]";
}

int popcount_status(uint32_t st) {
  int n = 0;
  for (uint32_t b = krb::kStatusRsWait; b <= krb::kStatusFlagWait; b <<= 1)
    if (st & b) ++n;
  return n;
}

// Result JSON of one engine, same fields as the reference's ResultJson
// (qwen_main.cpp:1785-1803) plus B200 extras.
std::string stage_json(krb::Engine &e, const std::string &mode, int warmup, int iters,
                       const std::vector<double> &samples, const std::vector<double> &host,
                       const krb::Engine::Verdict &v, uint32_t status, int flag_edges) {
  double best, typ, hb, ht;
  stats(samples, &best, &typ);
  stats(host, &hb, &ht);
  std::ostringstream os;
  os << "{\"mode\":\"" << mode << "\",\"seq\":" << e.cfg().seq << ",\"device\":" << e.device()
     << ",\"warmup\":" << warmup << ",\"iters\":" << iters << ",\"best_us\":" << fmt(best)
     << ",\"typical_us\":" << fmt(typ) << ",\"samples_us\":" << samples_json(samples)
     << ",\"argmax\":" << v.argmax << ",\"ref_argmax\":" << v.ref_argmax
     << ",\"maxdiff\":" << v.maxdiff << ",\"abs_mean\":" << v.abs_mean
     << ",\"flag_edges\":" << flag_edges << ",\"flag_timeouts\":" << popcount_status(status)
     << ",\"host_best_us\":" << fmt(hb) << ",\"host_typical_us\":" << fmt(ht)
     << ",\"status\":" << status << ",\"rank\":" << e.rank() << ",\"world\":" << e.world()
     << ",\"has_ref\":" << (v.has_ref ? "true" : "false") << "}";
  return os.str();
}

}  // namespace

// =================================================================== reference ABI
KRB_EXPORT const char *kr_version(void) { return "KernRelay 0.3 (libkernrelay, B200 sm_100a)"; }

KRB_EXPORT int kr_plan_run(const char *schedule_json, int iters, int warmup, const char *devices,
                           const char *mode, const char *out_json) {
  if (!schedule_json || !out_json) return 2;  // kr_api.cpp:27
  try {
    const std::string res = krb::plan::run(schedule_json, iters, warmup, devices ? devices : "",
                                           mode ? mode : "direct", out_json);
    std::printf("%s\n", res.c_str());  // the reference prints its result line too
    std::fflush(stdout);
    return 0;
  } catch (const std::exception &e) {
    g_last_error = e.what();
    std::ofstream f(out_json);
    f << "{\"error\":\"" << krb::json::escape(e.what()) << "\"}\n";
    return 1;
  }
}

KRB_EXPORT int kr_qwen_run(const char *model_dir, const char *mode, int seq, int device,
                           int warmup, int iters, char *out, size_t out_cap) {
  try {
    if (!model_dir || !*model_dir) throw std::runtime_error("model path required");
    krb::EngineOpts o;
    o.model_dir = model_dir;
    o.mode = mode ? mode : "serial_graph";
    o.seq = seq;
    o.device = device;
    o.tiles = 4;
    if (const char *t = std::getenv("KR_TILES")) o.tiles = std::max(1, std::atoi(t));
    krb::Engine e(o);
    if (e.mode().tp) throw std::runtime_error("use kr_qwen_tp_run for tp modes");
    e.run();
    e.sync();
    krb::Engine::Verdict v = e.verify();
    if (e.mode().graph) e.capture_graph();
    for (int i = 0; i < warmup; ++i) {
      e.run();
      e.sync();
    }
    std::vector<double> samples, host;
    for (int i = 0; i < std::max(1, iters); ++i) {
      e.sync();
      const auto t0 = Clock::now();
      e.run();
      const auto th = Clock::now();
      e.sync();
      const auto t1 = Clock::now();
      samples.push_back(us_between(t0, t1));
      host.push_back(us_between(t0, th));
    }
    v = e.verify();  // after replays, re-check numerics (qwen_main.cpp:2168)
    const uint32_t st = e.read_status();
    if (st) throw std::runtime_error("device status " + std::to_string(st));
    return write_out(stage_json(e, o.mode, warmup, iters, samples, host, v, st,
                                e.mode().split ? e.cfg().L * o.tiles : 0),
                     out, out_cap);
  } catch (const std::exception &ex) {
    return write_error(ex.what(), out, out_cap);
  }
}

// PP=2 layer pipeline (qwen_main.cpp:1359-1528 BuildPP, 1993-2146 RunQwenPP):
// stage 0 on dev0 runs embed + layers [0, L/2), stage 1 on dev1 layers [L/2, L) +
// final norm + lm_head.  Per request r the stage-0 residual stream (fp32 [S, H])
// crosses NVLink by one peer copy into stage 1's receive buffer r; a cross-device
// event orders stage 1 after the copy (the reference's HcclSend/HcclRecv).
// "pp"/"pp1": all requests are enqueued back to back, so stage 0 computes request
// r+1 while stage 1 computes request r; "pp_serial"/"pp1_serial": stage 0 starts
// request r only after stage 1 finished request r-1 (the no-overlap baseline).
// Both stages are driven from this thread (stage 0 then stage 1 per request), so
// every cross-device wait refers to the current iteration's record.
KRB_EXPORT int kr_qwen_pp_run(const char *model_dir, const char *mode, int seq, int dev0,
                              int dev1, int requests, int warmup, int iters, char *out,
                              size_t out_cap) {
  std::vector<void *> recv;
  std::vector<cudaEvent_t> ev_sent, ev_done;
  std::unique_ptr<krb::Engine> eng[2];
  auto cleanup = [&] {
    for (auto &e : ev_sent) if (e) cudaEventDestroy(e);
    for (auto &e : ev_done) if (e) cudaEventDestroy(e);
    if (!recv.empty()) {
      cudaSetDevice(dev1);
      for (void *p : recv) if (p) cudaFree(p);
    }
    recv.clear();
    ev_sent.clear();
    ev_done.clear();
    eng[0].reset();
    eng[1].reset();
  };
  try {
    if (!model_dir || !*model_dir) throw std::runtime_error("model path required");
    const std::string mname = mode ? mode : "pp";
    const krb::Mode m = krb::Mode::parse(mname);
    if (!m.pp) throw std::runtime_error("kr_qwen_pp_run needs a pp mode (pp, pp_serial, pp1, pp1_serial)");
    if (dev1 < 0 || dev1 == dev0) throw std::runtime_error("--device2 must be a different device");
    if (requests < 1 || requests > 8) throw std::runtime_error("--requests must be in 1..8");
    int ndev = 0;
    KRB_CUDA(cudaGetDeviceCount(&ndev));
    if (dev0 < 0 || dev0 >= ndev || dev1 >= ndev) throw std::runtime_error("device not present");
    const int devs[2] = {dev0, dev1};
    for (int i = 0; i < 2; ++i) {
      int can = 0;
      KRB_CUDA(cudaDeviceCanAccessPeer(&can, devs[i], devs[1 - i]));
      if (!can) throw std::runtime_error("no peer access between the two devices");
      KRB_CUDA(cudaSetDevice(devs[i]));
      cudaError_t r = cudaDeviceEnablePeerAccess(devs[1 - i], 0);
      if (r == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else KRB_CUDA(r);
    }
    {
      std::string errs[2];
      std::vector<std::thread> th;
      for (int st = 0; st < 2; ++st)
        th.emplace_back([&, st] {
          try {
            krb::EngineOpts o;
            o.model_dir = model_dir;
            o.mode = mname;
            o.seq = seq;
            o.device = devs[st];
            o.pp_stage = st;
            o.pp_stages = 2;
            eng[st] = std::make_unique<krb::Engine>(o);
          } catch (const std::exception &ex) {
            errs[st] = ex.what();
          }
        });
      for (auto &t : th) t.join();
      for (int st = 0; st < 2; ++st)
        if (!errs[st].empty()) throw std::runtime_error("stage" + std::to_string(st) + ": " + errs[st]);
    }
    const size_t bytes = size_t(seq) * eng[0]->cfg().H * 4;
    recv.assign(requests, nullptr);
    ev_sent.assign(requests, nullptr);
    ev_done.assign(requests, nullptr);
    KRB_CUDA(cudaSetDevice(dev1));
    for (int r = 0; r < requests; ++r) {
      KRB_CUDA(cudaMalloc(&recv[r], bytes));
      KRB_CUDA(cudaEventCreateWithFlags(&ev_done[r], cudaEventDisableTiming));
    }
    KRB_CUDA(cudaSetDevice(dev0));
    for (int r = 0; r < requests; ++r)
      KRB_CUDA(cudaEventCreateWithFlags(&ev_sent[r], cudaEventDisableTiming));
    krb::Engine &s0 = *eng[0];
    krb::Engine &s1 = *eng[1];
    auto iteration = [&] {
      for (int r = 0; r < requests; ++r) {
        KRB_CUDA(cudaSetDevice(dev0));
        if (!m.pp_pipeline && r > 0) KRB_CUDA(cudaStreamWaitEvent(s0.stream(), ev_done[r - 1], 0));
        s0.enqueue_stage(nullptr);
        KRB_CUDA(cudaMemcpyPeerAsync(recv[r], dev1, s0.residual_out(), dev0, bytes, s0.stream()));
        KRB_CUDA(cudaEventRecord(ev_sent[r], s0.stream()));
        KRB_CUDA(cudaSetDevice(dev1));
        KRB_CUDA(cudaStreamWaitEvent(s1.stream(), ev_sent[r], 0));
        s1.enqueue_stage(static_cast<const float *>(recv[r]));
        KRB_CUDA(cudaEventRecord(ev_done[r], s1.stream()));
      }
      s0.sync();
      s1.sync();
    };
    // first run (correctness, outside the timing), warm-up, timed iterations
    iteration();
    krb::Engine::Verdict v = s1.verify();
    for (int w = 0; w < warmup; ++w) iteration();
    std::vector<double> wall;
    for (int i = 0; i < std::max(1, iters); ++i) {
      const auto t0 = Clock::now();
      iteration();
      wall.push_back(us_between(t0, Clock::now()));
    }
    v = s1.verify();
    uint32_t st0 = s0.read_status(), st1 = s1.read_status();
    if (st0 || st1)
      throw std::runtime_error("device status " + std::to_string(st0) + "/" + std::to_string(st1));
    const krb::Engine::Verdict none;
    const std::string j0 = stage_json(s0, "pp_stage0", warmup, iters, wall, {}, none, st0, 0);
    const std::string j1 = stage_json(s1, "pp_stage1", warmup, iters, wall, {}, v, st1, 0);
    double best, typ;
    stats(wall, &best, &typ);
    std::ostringstream os;
    os << "{\"mode\":\"" << (m.pp_pipeline ? "pp_pipeline" : "pp_serial") << "\",\"seq\":" << seq
       << ",\"requests\":" << requests << ",\"devices\":[" << dev0 << "," << dev1 << "]"
       << ",\"layers\":[[" << s0.layer_begin() << "," << s0.layer_end() << "],["
       << s1.layer_begin() << "," << s1.layer_end() << "]]"
       << ",\"wall_best_us\":" << fmt(best) << ",\"wall_typical_us\":" << fmt(typ)
       << ",\"wall_samples_us\":" << samples_json(wall) << ",\"stages\":[" << j0 << "," << j1
       << "]}";
    cleanup();
    return write_out(os.str(), out, out_cap);
  } catch (const std::exception &ex) {
    cudaDeviceSynchronize();
    cleanup();
    return write_error(ex.what(), out, out_cap);
  }
}

namespace {

std::vector<int> tp_devices(int k, int dev0, int dev1) {
  std::vector<int> d;
  if (const char *e = std::getenv("KR_TP_DEVICES")) {
    std::stringstream ss(e);
    std::string tok;
    while (std::getline(ss, tok, ','))
      if (!tok.empty()) d.push_back(std::atoi(tok.c_str()));
    if (int(d.size()) < k) throw std::runtime_error("KR_TP_DEVICES lists fewer devices than k");
    d.resize(k);
  } else if (k == 2) {
    if (dev1 < 0 || dev1 == dev0) throw std::runtime_error("--device2 must be a different device");
    d = {dev0, dev1};
  } else {
    for (int i = 0; i < k; ++i) d.push_back(dev0 + i);
  }
  for (size_t i = 0; i < d.size(); ++i)
    for (size_t j = i + 1; j < d.size(); ++j)
      if (d[i] == d[j]) throw std::runtime_error("tp devices must be distinct");
  return d;
}

}  // namespace

KRB_EXPORT int kr_qwen_tp_run(const char *model_dir, const char *mode, int seq, int dev0,
                              int dev1, int tiles, int warmup, int iters, char *out,
                              size_t out_cap) {
  try {
    if (!model_dir || !*model_dir) throw std::runtime_error("model path required");
    const std::string mname = mode ? mode : "tp2";
    const krb::Mode m = krb::Mode::parse(mname);
    if (!m.tp) throw std::runtime_error("kr_qwen_tp_run needs a tp mode");
    if (tiles < 1 || tiles > 8) throw std::runtime_error("--tiles must be in 1..8");
    const int k = m.world;
    const int t_eff = m.split ? tiles : 1;
    const std::vector<int> devs = tp_devices(k, dev0, dev1);
    int ndev = 0;
    KRB_CUDA(cudaGetDeviceCount(&ndev));
    for (int d : devs)
      if (d < 0 || d >= ndev) throw std::runtime_error("device " + std::to_string(d) + " not present");
    // peer access between all pairs (NVLink/NVSwitch)
    if (m.split && k > 1) {
      for (int i : devs)
        for (int j : devs) {
          if (i == j) continue;
          int can = 0;
          KRB_CUDA(cudaDeviceCanAccessPeer(&can, i, j));
          if (!can) throw std::runtime_error("no peer access between devices");
          KRB_CUDA(cudaSetDevice(i));
          cudaError_t r = cudaDeviceEnablePeerAccess(j, 0);
          if (r == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
          else KRB_CUDA(r);
        }
    }
    // build the engines in parallel (weight load dominates)
    std::vector<std::unique_ptr<krb::Engine>> eng(k);
    std::vector<std::string> errs(k);
    {
      std::vector<std::thread> th;
      for (int r = 0; r < k; ++r)
        th.emplace_back([&, r] {
          try {
            krb::EngineOpts o;
            o.model_dir = model_dir;
            o.mode = mname;
            o.seq = seq;
            o.rank = r;
            o.world = k;
            o.device = devs[r];
            o.tiles = t_eff;
            eng[r] = std::make_unique<krb::Engine>(o);
          } catch (const std::exception &ex) {
            errs[r] = ex.what();
          }
        });
      for (auto &t : th) t.join();
      for (int r = 0; r < k; ++r)
        if (!errs[r].empty()) throw std::runtime_error("rank" + std::to_string(r) + ": " + errs[r]);
    }
    std::vector<ncclComm_t> comms(k, nullptr);
    if (m.split) {
      std::vector<void *> bases(k);
      for (int r = 0; r < k; ++r) bases[r] = eng[r]->sym_base();
      for (int r = 0; r < k; ++r) eng[r]->set_peers(bases);
    } else if (k > 1) {
      if (ncclCommInitAll(comms.data(), k, devs.data()) != ncclSuccess)
        throw std::runtime_error("ncclCommInitAll failed");
      for (int r = 0; r < k; ++r) eng[r]->set_nccl(comms[r]);
    }
    std::barrier<> bar(k + 1);  // the k workers and the timing thread
    std::mutex mu;
    std::string err;
    std::vector<std::string> stage(k);
    std::vector<double> wall;
    auto worker = [&](int r) {
      krb::Engine &e = *eng[r];
      bool ok = true;
      auto guard = [&](auto fn) {
        if (!ok) return;
        try {
          fn();
        } catch (const std::exception &ex) {
          ok = false;
          std::lock_guard<std::mutex> lk(mu);
          if (err.empty()) err = "rank" + std::to_string(r) + ": " + ex.what();
        }
      };
      krb::Engine::Verdict v;
      guard([&] {
        KRB_CUDA(cudaSetDevice(e.device()));
        e.run();
        e.sync();
        v = e.verify();
        if (e.mode().graph) e.capture_graph();
      });
      bar.arrive_and_wait();
      for (int w = 0; w < warmup; ++w) {
        bar.arrive_and_wait();
        guard([&] {
          e.run();
          e.sync();
        });
        bar.arrive_and_wait();
      }
      std::vector<double> samples;
      for (int i = 0; i < std::max(1, iters); ++i) {
        bar.arrive_and_wait();
        const auto t0 = Clock::now();
        guard([&] {
          e.run();
          e.sync();
        });
        samples.push_back(us_between(t0, Clock::now()));
        bar.arrive_and_wait();
      }
      guard([&] {
        v = e.verify();
        const uint32_t st = e.read_status();
        if (st) throw std::runtime_error("device status " + std::to_string(st));
        stage[r] = stage_json(e, "tp_rank" + std::to_string(r), warmup, iters, samples, {}, v, st,
                              e.mode().split ? e.cfg().L * t_eff : 0);
      });
      bar.arrive_and_wait();
    };
    std::vector<std::thread> th;
    for (int r = 0; r < k; ++r) th.emplace_back(worker, r);
    bar.arrive_and_wait();  // first run + verify done
    for (int w = 0; w < warmup; ++w) {
      bar.arrive_and_wait();
      bar.arrive_and_wait();
    }
    for (int i = 0; i < std::max(1, iters); ++i) {
      bar.arrive_and_wait();
      const auto t0 = Clock::now();
      bar.arrive_and_wait();
      wall.push_back(us_between(t0, Clock::now()));
    }
    bar.arrive_and_wait();
    for (auto &t : th) t.join();
    eng.clear();  // graphs that hold NCCL work go before the communicators
    for (int r = 0; r < k; ++r) {
      if (comms[r]) ncclCommDestroy(comms[r]);
    }
    if (!err.empty()) throw std::runtime_error(err);
    double best, typ;
    stats(wall, &best, &typ);
    std::ostringstream os;
    os << "{\"mode\":\"" << mname << "\",\"seq\":" << seq << ",\"tiles\":" << t_eff << ",\"k\":" << k
       << ",\"devices\":[";
    for (int r = 0; r < k; ++r) os << (r ? "," : "") << devs[r];
    os << "],\"wall_best_us\":" << fmt(best) << ",\"wall_typical_us\":" << fmt(typ)
       << ",\"wall_samples_us\":" << samples_json(wall) << ",\"stages\":[";
    for (int r = 0; r < k; ++r) os << (r ? "," : "") << stage[r];
    os << "]}";
    return write_out(os.str(), out, out_cap);
  } catch (const std::exception &ex) {
    return write_error(ex.what(), out, out_cap);
  }
}


// =================================================================== B200 extensions
KRB_EXPORT const char *krb_last_error(void) { return g_last_error.c_str(); }

KRB_EXPORT int krb_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

KRB_EXPORT int krb_synth_normal_host(const char *name, uint64_t seed, double std_, double mean,
                                     uint64_t offset, uint64_t n, uint16_t *out) {
  try {
    if (!name || !out) throw std::runtime_error("null argument");
    const uint64_t key = krb::synth_key(name, seed);
    const double scale = krb::synth_scale(std_);
    const unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t)
      th.emplace_back([=] {
        const uint64_t lo = n * t / nt, hi = n * (t + 1) / nt;
        for (uint64_t i = lo; i < hi; ++i)
          out[i] = krb::synth_normal_bf16(key, offset + i, scale, mean);
      });
    for (auto &x : th) x.join();
    return 0;
  } catch (const std::exception &e) {
    return fail(e);
  }
}

#define KRB_OP_BEGIN try {
#define KRB_OP_END      \
  return 0;             \
  }                     \
  catch (const std::exception &e) { return fail(e); }

using bf = __nv_bfloat16;

KRB_EXPORT int krb_gemm_bf16(const void *A, long lda, const void *B, long ldb, void *C, long ldc,
                             const void *bias, int M, int N, int K, int bn, void *stream) {
  KRB_OP_BEGIN
  krb::gemm_bf16(static_cast<const bf *>(A), lda, static_cast<const bf *>(B), ldb,
                 static_cast<bf *>(C), ldc, static_cast<const bf *>(bias), M, N, K, bn, 0, nullptr,
                 as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_gemm_qkv_rope_bf16(const void *A, long lda, const void *B, long ldb, void *C,
                                      long ldc, const void *bias, int M, int K, int HQ, int HKV,
                                      int D, const void *cos_tab, const void *sin_tab,
                                      const void *q_norm, const void *k_norm, float eps,
                                      void *vt, long ldvt, void *stream) {
  KRB_OP_BEGIN
  krb::gemm_qkv_rope_bf16(static_cast<const bf *>(A), lda, static_cast<const bf *>(B), ldb,
                          static_cast<bf *>(C), ldc, static_cast<const bf *>(bias), M, K, HQ, HKV, D,
                          static_cast<const bf *>(cos_tab), static_cast<const bf *>(sin_tab),
                          static_cast<const bf *>(q_norm), static_cast<const bf *>(k_norm), eps,
                          nullptr, as_stream(stream), static_cast<__half *>(vt), ldvt);
  KRB_OP_END
}

KRB_EXPORT int krb_gemm_silu_bf16(const void *A, long lda, const void *Bgu, long ldb, void *act,
                                  long ldact, int M, int n_out, int K, int bn, void *stream) {
  KRB_OP_BEGIN
  if (bn != 128 && bn != 192 && bn != 256)
    throw std::runtime_error("gemm_silu: bn must be 128, 192 or 256");
  krb::gemm_silu_bf16(static_cast<const bf *>(A), lda, static_cast<const bf *>(Bgu), ldb,
                      static_cast<bf *>(act), ldact, M, n_out, K, bn, 0, nullptr, as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_rmsnorm_bf16(const void *x, const void *gamma, void *y, float *rstd, int rows,
                                int H, float eps, void *stream) {
  KRB_OP_BEGIN
  krb::rmsnorm_bf16(static_cast<const bf *>(x), static_cast<const bf *>(gamma), static_cast<bf *>(y),
                    rstd, rows, H, eps, as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_add_rmsnorm_bf16(const void *a, const void *b, const void *gamma, void *y,
                                    float *rstd, void *sum, int rows, int H, float eps,
                                    void *stream) {
  KRB_OP_BEGIN
  krb::add_rmsnorm_bf16(static_cast<const bf *>(a), static_cast<const bf *>(b),
                        static_cast<const bf *>(gamma), static_cast<bf *>(y), rstd,
                        static_cast<bf *>(sum), rows, H, eps, as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_gemm_f32out(const void *A, long lda, const void *B, long ldb, float *out,
                               long ld, int M, int N, int K, int bn, void *stream) {
  KRB_OP_BEGIN
  krb::gemm_f32out(static_cast<const bf *>(A), lda, static_cast<const bf *>(B), ldb, out, ld, M, N,
                   K, bn, nullptr, as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_add_rmsnorm_res_f32(const float *res, const void *delta, const void *gamma,
                                       void *y, float *sum, int rows, int H, float eps,
                                       void *stream) {
  KRB_OP_BEGIN
  krb::add_rmsnorm_res_f32(res, static_cast<const bf *>(delta), static_cast<const bf *>(gamma),
                           static_cast<bf *>(y), sum, rows, H, eps, as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_embed_bf16(const int64_t *ids, const void *table, void *out, int S, int H, int V,
                              uint32_t *status, void *stream) {
  KRB_OP_BEGIN
  krb::embed_bf16(ids, static_cast<const bf *>(table), static_cast<bf *>(out), S, H, V, status,
                  as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_qk_norm_rope_bf16(void *qkv, int S, int HQ, int HKV, int D, const void *cos_tab,
                                     const void *sin_tab, const void *q_norm, const void *k_norm,
                                     float eps, void *stream) {
  KRB_OP_BEGIN
  krb::qk_norm_rope_bf16(static_cast<bf *>(qkv), S, HQ, HKV, D, static_cast<const bf *>(cos_tab),
                         static_cast<const bf *>(sin_tab), static_cast<const bf *>(q_norm),
                         static_cast<const bf *>(k_norm), eps, as_stream(stream));
  KRB_OP_END
}

KRB_EXPORT int krb_attention_prefill_bf16(const void *qkv, void *out, int S, int HQ, int HKV, int D,
                                          float scale, int impl, uint32_t *status, void *stream) {
  KRB_OP_BEGIN
  // impl 0 / 2: the tcgen05 kernel (the only attention of this build; 1 was mma.sync)
  if (impl != 0 && impl != 2) throw std::runtime_error("attention: impl must be 0 or 2 (tcgen05)");
  // V^T scratch, stream-ordered: allocated and released on the caller's stream
  cudaStream_t s = as_stream(stream);
  const long ldv = (long(S) + 7) / 8 * 8;
  void *vt = nullptr;
  KRB_CUDA(cudaMallocAsync(&vt, size_t(HKV) * D * ldv * 2, s));
  try {
    krb::attention_vt(static_cast<const bf *>(qkv), static_cast<__half *>(vt), ldv, S, HQ, HKV, D, s);
    krb::attention_tc_bf16(static_cast<const bf *>(qkv), static_cast<const __half *>(vt), ldv,
                           static_cast<bf *>(out), S, HQ, HKV, D, scale, status, s);
  } catch (...) {
    cudaFreeAsync(vt, s);
    throw;
  }
  KRB_CUDA(cudaFreeAsync(vt, s));
  KRB_OP_END
}

KRB_EXPORT int krb_relay_down_single(const void *act, const void *w_down, const void *resid,
                                     const void *gamma, void *sum_out, void *x_out, int S, int H,
                                     int K, int tiles, float eps, int bn, uint32_t *status,
                                     void *stream) {
  void *scratch = nullptr;
  try {
    if (tiles < 1 || S % tiles) throw std::runtime_error("relay: S % tiles != 0");
    const int dev_bn = bn > 0 ? bn : 256;
    krb::SymLayout L = krb::SymLayout::make(S, H, tiles, 1);
    cudaStream_t s = as_stream(stream);
    KRB_CUDA(cudaMalloc(&scratch, L.bytes));
    KRB_CUDA(cudaMemsetAsync(scratch, 0, L.bytes, s));
    // epoch = 1 for this single run
    krb::bump_epoch(reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(scratch) + L.epoch()), s);
    krb::RelayArgs ra{};
    ra.S = S;
    ra.H = H;
    ra.K = K;
    ra.T = tiles;
    ra.k = 1;
    ra.rank = 0;
    ra.R = S / tiles;
    ra.Rk = ra.R;
    ra.nseg = (H + 255) / 256;
    ra.peer_base[0] = static_cast<uint8_t *>(scratch);
    ra.local_base = static_cast<uint8_t *>(scratch);
    ra.part_off = L.part_off;
    ra.red_off = L.red_off;
    ra.flag_off = L.flag_off;
    ra.epoch = reinterpret_cast<const uint32_t *>(static_cast<uint8_t *>(scratch) + L.epoch());
    ra.layer = 0;
    ra.L = 1;
    ra.resid = static_cast<const float *>(resid);
    ra.gamma = static_cast<const bf *>(gamma);
    ra.sum_out = static_cast<float *>(sum_out);
    ra.x_out = static_cast<bf *>(x_out);
    ra.eps = eps;
    ra.do_norm = 1;
    ra.timeout_ns = 2000000000ull;
    ra.status = status;
    ra.trace = nullptr;
    krb::relay_down_layer(static_cast<const bf *>(act), K, static_cast<const bf *>(w_down), K, dev_bn,
                          ra, s);
    KRB_CUDA(cudaStreamSynchronize(s));
    KRB_CUDA(cudaFree(scratch));
    return 0;
  } catch (const std::exception &e) {
    if (scratch) {
      cudaDeviceSynchronize();
      cudaFree(scratch);
    }
    return fail(e);
  }
}

// Allocation-free form of krb_relay_down_single: the relay's counters live in a
// static device array (relay.cu), looked up once per device; nothing is allocated
// or freed and the stream is not synchronised.
KRB_EXPORT int krb_relay_down_single_noalloc(const void *act, const void *w_down,
                                             const void *resid, const void *gamma, void *sum_out,
                                             void *x_out, int S, int H, int K, int tiles,
                                             float eps, int bn, uint32_t *status, void *stream) {
  try {
    if (tiles < 1 || S % tiles) throw std::runtime_error("relay: S % tiles != 0");
    const krb::SymLayout L = krb::SymLayout::flags_only(tiles);
    if (L.bytes > krb::kRelayNoAllocScratchBytes)
      throw std::runtime_error("relay (no-alloc): " + std::to_string(tiles) + " row tiles need " +
                               std::to_string(L.bytes) + " bytes of scratch; the static scratch "
                               "holds " + std::to_string(krb::kRelayNoAllocScratchBytes) +
                               " bytes (at most 127 row tiles)");
    const int dev_bn = bn > 0 ? bn : 256;
    cudaStream_t s = as_stream(stream);
    uint8_t *scratch = krb::relay_noalloc_scratch();
    // the counters and the epoch must start at zero; epoch = 1 for this run
    KRB_CUDA(cudaMemsetAsync(scratch, 0, L.bytes, s));
    krb::bump_epoch(reinterpret_cast<uint32_t *>(scratch + L.epoch()), s);
    krb::RelayArgs ra{};
    ra.S = S;
    ra.H = H;
    ra.K = K;
    ra.T = tiles;
    ra.k = 1;
    ra.rank = 0;
    ra.R = S / tiles;
    ra.Rk = ra.R;
    ra.nseg = (H + 255) / 256;
    ra.peer_base[0] = scratch;
    ra.local_base = scratch;
    ra.part_off = L.part_off;
    ra.red_off = L.red_off;
    ra.flag_off = L.flag_off;
    ra.epoch = reinterpret_cast<const uint32_t *>(scratch + L.epoch());
    ra.layer = 0;
    ra.L = 1;
    ra.resid = static_cast<const float *>(resid);
    ra.gamma = static_cast<const bf *>(gamma);
    ra.sum_out = static_cast<float *>(sum_out);
    ra.x_out = static_cast<bf *>(x_out);
    ra.eps = eps;
    ra.do_norm = 1;
    ra.timeout_ns = 2000000000ull;
    ra.status = status;
    ra.trace = nullptr;
    krb::relay_down_layer(static_cast<const bf *>(act), K, static_cast<const bf *>(w_down), K, dev_bn,
                          ra, s);
    return 0;
  } catch (const std::exception &e) {
    return fail(e);
  }
}

// Failure-detection probe: rank 0 of a two-rank relay whose peer never runs.
// The "peer" region is a second local allocation nobody signals, so rank 0's
// bounded waits for the peer's partials must expire after `timeout_ms`, set
// the status bits and return with the context intact.
KRB_EXPORT int krb_relay_timeout_probe(int S, int H, int K, int tiles, float timeout_ms,
                                       uint32_t *status_out) {
  void *mine = nullptr, *ghost = nullptr, *bufs = nullptr;
  try {
    if (!status_out) throw std::runtime_error("null status");
    const int k = 2;
    krb::SymLayout L = krb::SymLayout::make(S, H, tiles, k);
    KRB_CUDA(cudaMalloc(&mine, L.bytes));
    KRB_CUDA(cudaMalloc(&ghost, L.bytes));
    const size_t act_b = size_t(S) * K * 2, w_b = size_t(H) * K * 2, res_b = size_t(S) * H * 4;
    KRB_CUDA(cudaMalloc(&bufs, act_b + w_b + 2 * res_b + size_t(S) * H * 2 + H * 2 + 256));
    KRB_CUDA(cudaMemset(mine, 0, L.bytes));
    KRB_CUDA(cudaMemset(ghost, 0, L.bytes));
    KRB_CUDA(cudaMemset(bufs, 0, act_b + w_b + 2 * res_b + size_t(S) * H * 2 + H * 2 + 256));
    uint8_t *p = static_cast<uint8_t *>(bufs);
    const bf *act = reinterpret_cast<const bf *>(p);
    const bf *w = reinterpret_cast<const bf *>(p + act_b);
    float *res = reinterpret_cast<float *>(p + act_b + w_b);
    float *sum = reinterpret_cast<float *>(p + act_b + w_b + res_b);
    bf *x = reinterpret_cast<bf *>(p + act_b + w_b + 2 * res_b);
    bf *gamma = reinterpret_cast<bf *>(p + act_b + w_b + 2 * res_b + size_t(S) * H * 2);
    uint32_t *status = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(gamma) + H * 2);
    krb::bump_epoch(reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(mine) + L.epoch()), nullptr);
    krb::RelayArgs ra{};
    ra.S = S;
    ra.H = H;
    ra.K = K;
    ra.T = tiles;
    ra.k = k;
    ra.rank = 0;
    ra.R = S / tiles;
    ra.Rk = ra.R / k;
    ra.nseg = (H + 255) / 256;
    ra.peer_base[0] = static_cast<uint8_t *>(mine);
    ra.peer_base[1] = static_cast<uint8_t *>(ghost);
    ra.local_base = static_cast<uint8_t *>(mine);
    ra.part_off = L.part_off;
    ra.red_off = L.red_off;
    ra.flag_off = L.flag_off;
    ra.epoch = reinterpret_cast<const uint32_t *>(static_cast<uint8_t *>(mine) + L.epoch());
    ra.layer = 0;
    ra.L = 1;
    ra.resid = res;
    ra.gamma = gamma;
    ra.sum_out = sum;
    ra.x_out = x;
    ra.eps = 1e-6f;
    ra.do_norm = 1;
    ra.timeout_ns = uint64_t(double(timeout_ms) * 1e6);
    ra.status = status;
    // the engine's exchange path (fp16 operands; the buffers are zero, the same bits in
    // either format)
    krb::relay_down_layer(reinterpret_cast<const __half *>(act), K,
                          reinterpret_cast<const __half *>(w), K, 256, ra, nullptr);
    KRB_CUDA(cudaDeviceSynchronize());
    KRB_CUDA(cudaMemcpy(status_out, status, 4, cudaMemcpyDeviceToHost));
    cudaFree(mine);
    cudaFree(ghost);
    cudaFree(bufs);
    return 0;
  } catch (const std::exception &e) {
    cudaDeviceSynchronize();
    if (mine) cudaFree(mine);
    if (ghost) cudaFree(ghost);
    if (bufs) cudaFree(bufs);
    return fail(e);
  }
}

KRB_EXPORT int krb_plan_check(const char *schedule_json, char *out, size_t out_cap) {
  try {
    if (!schedule_json) throw std::runtime_error("schedule path required");
    return write_out(krb::plan::check(schedule_json), out, out_cap);
  } catch (const std::exception &e) {
    return write_error(e.what(), out, out_cap);
  }
}

KRB_EXPORT int krb_relay_plan(int S, int H, int tiles, int k, int rank, int bn, char *out,
                              size_t cap) {
  try {
    if (tiles < 1 || S % tiles || (S / tiles) % 128 || k < 1 || (S / tiles) % k || rank < 0 ||
        rank >= k || (bn != 128 && bn != 224 && bn != 256))
      throw std::runtime_error("relay plan: unsupported shape");
    // the SM count of the current device, or B200's 148 where no GPU is visible
    int grid = 148;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0) {
      int dev = 0;
      KRB_CUDA(cudaGetDevice(&dev));
      grid = krb::sm_count(dev);
    } else {
      cudaGetLastError();
    }
    const int cg = krb::relay_uses_pairs(S, tiles, bn) ? 2 : 1;
    const krb::TileSched ts = krb::relay_tile_sched(S, H, tiles, bn, grid, cg);
    const int R = S / tiles, Rk = R / k;
    std::ostringstream os;
    os << "{\"R\":" << R << ",\"Rk\":" << Rk << ",\"grid\":" << grid << ",\"bn\":" << bn
       << ",\"cta_group\":" << cg
       << ",\"bn2\":" << ts.bn2 << ",\"p1\":" << ts.p1 << ",\"total\":" << ts.total()
       << ",\"nseg\":" << (H + 255) / 256 << ",\"band_tiles\":[";
    for (int t = 0; t < tiles; ++t) os << (t ? "," : "") << ts.band_tiles(t);
    // the consumer's targets per run and layer: k = 1 every CTA's share of the GEMM tiles of
    // row tile t; k > 1 one forwarded signal per (row tile, source) and per (row tile, owner)
    os << "],\"rs_expect\":[";
    for (int t = 0; t < tiles; ++t) os << (t ? "," : "") << (k == 1 ? cg * ts.band_tiles(t) : 1);
    os << "],\"ag_expect\":" << (k == 1 ? 0 : 1) << ",\"tiles\":[";
    for (int i = 0; i < ts.total(); ++i) {
      int mb, n0, w;
      ts.tile(i, mb, n0, w);
      // [first 128-row block, 128-row blocks, first column, width]
      os << (i ? "," : "") << "[" << mb * cg << "," << cg << "," << n0 << "," << w << "]";
    }
    os << "],\"blocks\":[";
    for (int b = 0; b < S / 128; ++b) {
      const krb::RowRoute f = krb::relay_route(b * 128, R, Rk);
      const krb::RowRoute l = krb::relay_route(b * 128 + 127, R, Rk);
      os << (b ? "," : "") << "[" << f.tile << "," << f.owner << "," << l.owner << "]";
    }
    os << "]}";
    return write_out(os.str(), out, cap);
  } catch (const std::exception &e) {
    return write_error(e.what(), out, cap);
  }
}

// ---------------------------------------------------------------- per-rank engine
struct krb_engine {
  std::unique_ptr<krb::Engine> e;
  std::vector<void *> opened;  // IPC-mapped peer regions
  ncclComm_t comm = nullptr;
};

KRB_EXPORT int krb_microdag_create(int seq, int hidden, int intermediate, int tiles, int rank,
                                   int world, int device, const char *mode, uint64_t seed,
                                   krb_engine **out) {
  try {
    if (!mode || !out) throw std::runtime_error("null argument");
    krb::EngineOpts o;
    o.mode = mode;
    o.seq = seq;
    o.rank = rank;
    o.world = world;
    o.device = device;
    o.tiles = tiles;
    o.microdag = true;
    o.md_H = hidden;
    o.md_I = intermediate;
    o.md_seed = seed;
    auto *h = new krb_engine();
    try {
      h->e = std::make_unique<krb::Engine>(o);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
    return 0;
  } catch (const std::exception &e) {
    return fail(e);
  }
}

KRB_EXPORT int krb_engine_create(const char *model_dir, const char *mode, int seq, int rank,
                                 int world, int device, int tiles, krb_engine **out) {
  try {
    if (!model_dir || !mode || !out) throw std::runtime_error("null argument");
    krb::EngineOpts o;
    o.model_dir = model_dir;
    o.mode = mode;
    o.seq = seq;
    o.rank = rank;
    o.world = world;
    o.device = device;
    o.tiles = tiles;
    auto *h = new krb_engine();
    try {
      h->e = std::make_unique<krb::Engine>(o);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
    return 0;
  } catch (const std::exception &e) {
    return fail(e);
  }
}

KRB_EXPORT void krb_engine_destroy(krb_engine *h) {
  if (!h) return;
  if (h->e) cudaSetDevice(h->e->device());
  if (h->e) cudaStreamSynchronize(h->e->stream());
  h->e.reset();  // the engine's graph may hold NCCL work: release it first
  for (void *p : h->opened)
    if (p) cudaIpcCloseMemHandle(p);
  if (h->comm) ncclCommDestroy(h->comm);
  delete h;
}

KRB_EXPORT int krb_engine_ipc_handle(krb_engine *h, void *handle_out, size_t cap) {
  KRB_OP_BEGIN
  if (!h || !handle_out || cap < sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad argument");
  if (!h->e->sym_base()) throw std::runtime_error("engine has no relay region (not a split mode)");
  KRB_CUDA(cudaSetDevice(h->e->device()));
  cudaIpcMemHandle_t ipc;
  KRB_CUDA(cudaIpcGetMemHandle(&ipc, h->e->sym_base()));
  std::memcpy(handle_out, &ipc, sizeof(ipc));
  KRB_OP_END
}

KRB_EXPORT int krb_engine_open_peers(krb_engine *h, const void *handles, size_t bytes) {
  KRB_OP_BEGIN
  if (!h || !handles) throw std::runtime_error("bad argument");
  const int k = h->e->world();
  if (bytes < size_t(k) * sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("handle buffer too small");
  KRB_CUDA(cudaSetDevice(h->e->device()));
  std::vector<void *> bases(k, nullptr);
  for (int r = 0; r < k; ++r) {
    if (r == h->e->rank()) {
      bases[r] = h->e->sym_base();
      continue;
    }
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, static_cast<const char *>(handles) + size_t(r) * sizeof(ipc), sizeof(ipc));
    void *p = nullptr;
    KRB_CUDA(cudaIpcOpenMemHandle(&p, ipc, cudaIpcMemLazyEnablePeerAccess));
    h->opened.push_back(p);
    bases[r] = p;
  }
  h->e->set_peers(bases);
  KRB_OP_END
}

KRB_EXPORT int krb_nccl_unique_id(void *out, size_t cap) {
  KRB_OP_BEGIN
  if (!out || cap < sizeof(ncclUniqueId)) throw std::runtime_error("buffer too small");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) throw std::runtime_error("ncclGetUniqueId failed");
  std::memcpy(out, &id, sizeof(id));
  KRB_OP_END
}

KRB_EXPORT int krb_engine_init_nccl(krb_engine *h, const void *id, size_t bytes) {
  KRB_OP_BEGIN
  if (!h || !id || bytes < sizeof(ncclUniqueId)) throw std::runtime_error("bad argument");
  KRB_CUDA(cudaSetDevice(h->e->device()));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = ncclCommInitRank(&h->comm, h->e->world(), uid, h->e->rank());
  if (r != ncclSuccess) throw std::runtime_error(std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
  h->e->set_nccl(h->comm);
  KRB_OP_END
}

// In-process wiring of k engines (one per device, ranks 0..k-1 in order): peer
// access between every pair and direct peer pointers to the relay regions.
KRB_EXPORT int krb_engines_link(krb_engine **hs, int n) {
  KRB_OP_BEGIN
  if (!hs || n < 1 || n > krb::kMaxRanks) throw std::runtime_error("bad engine list");
  std::vector<void *> bases(n);
  for (int r = 0; r < n; ++r) {
    if (!hs[r] || hs[r]->e->rank() != r || hs[r]->e->world() != n)
      throw std::runtime_error("engines must be ranks 0..n-1 of one tp group");
    bases[r] = hs[r]->e->sym_base();
  }
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) {
      if (i == j) continue;
      const int di = hs[i]->e->device(), dj = hs[j]->e->device();
      int can = 0;
      KRB_CUDA(cudaDeviceCanAccessPeer(&can, di, dj));
      if (!can) throw std::runtime_error("no peer access between devices");
      KRB_CUDA(cudaSetDevice(di));
      cudaError_t r = cudaDeviceEnablePeerAccess(dj, 0);
      if (r == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else KRB_CUDA(r);
    }
  for (int r = 0; r < n; ++r) hs[r]->e->set_peers(bases);
  KRB_OP_END
}

// In-process NCCL communicators for k engines (ncclCommInitAll).
KRB_EXPORT int krb_engines_init_nccl(krb_engine **hs, int n) {
  KRB_OP_BEGIN
  if (!hs || n < 1 || n > krb::kMaxRanks) throw std::runtime_error("bad engine list");
  std::vector<int> devs(n);
  std::vector<ncclComm_t> comms(n, nullptr);
  for (int r = 0; r < n; ++r) devs[r] = hs[r]->e->device();
  if (ncclCommInitAll(comms.data(), n, devs.data()) != ncclSuccess)
    throw std::runtime_error("ncclCommInitAll failed");
  for (int r = 0; r < n; ++r) {
    hs[r]->comm = comms[r];
    hs[r]->e->set_nccl(comms[r]);
  }
  KRB_OP_END
}

KRB_EXPORT int krb_engine_capture(krb_engine *h) {
  KRB_OP_BEGIN
  h->e->capture_graph();
  KRB_OP_END
}

KRB_EXPORT int krb_engine_run(krb_engine *h) {
  KRB_OP_BEGIN
  h->e->run();
  KRB_OP_END
}

KRB_EXPORT int krb_engine_run_host(krb_engine *h, const int64_t *ids_host, float *logits_host) {
  KRB_OP_BEGIN
  h->e->enqueue_host(ids_host, logits_host);
  KRB_OP_END
}

KRB_EXPORT int krb_engine_sync(krb_engine *h) {
  KRB_OP_BEGIN
  h->e->sync();
  KRB_OP_END
}

KRB_EXPORT int krb_engine_stream(krb_engine *h, void **stream_out) {
  KRB_OP_BEGIN
  *stream_out = reinterpret_cast<void *>(h->e->stream());
  KRB_OP_END
}

KRB_EXPORT int krb_engine_status(krb_engine *h, uint32_t *status_out) {
  KRB_OP_BEGIN
  *status_out = h->e->read_status();
  KRB_OP_END
}

KRB_EXPORT int krb_engine_stage_times(krb_engine *h, char *out, size_t cap) {
  try {
    krb::StageTimes st = h->e->instrumented_run();
    std::ostringstream os;
    os << "{\"stage_us\":{\"embed\":" << fmt(st.embed) << ",\"qkv\":" << fmt(st.qkv)
       << ",\"rope\":" << fmt(st.rope) << ",\"attention\":" << fmt(st.attn) << ",\"o\":" << fmt(st.o)
       << ",\"addnorm\":" << fmt(st.addnorm) << ",\"gateup\":" << fmt(st.gateup)
       << ",\"down\":" << fmt(st.down) << ",\"allreduce\":" << fmt(st.allreduce)
       << ",\"addnorm2\":" << fmt(st.addnorm2) << ",\"relay\":" << fmt(st.relay)
       << ",\"lm_head\":" << fmt(st.lm_head) << "},\"total_us\":" << fmt(st.total) << "}";
    return write_out(os.str(), out, cap);
  } catch (const std::exception &e) {
    return write_error(e.what(), out, cap);
  }
}

KRB_EXPORT int krb_engine_verify(krb_engine *h, char *out, size_t cap) {
  try {
    krb::Engine::Verdict v = h->e->verify();
    std::ostringstream os;
    os << "{\"argmax\":" << v.argmax << ",\"ref_argmax\":" << v.ref_argmax << ",\"maxdiff\":" << v.maxdiff
       << ",\"abs_mean\":" << v.abs_mean << ",\"has_ref\":" << (v.has_ref ? "true" : "false") << "}";
    return write_out(os.str(), out, cap);
  } catch (const std::exception &e) {
    return write_error(e.what(), out, cap);
  }
}

KRB_EXPORT int krb_engine_last_logits(krb_engine *h, float *out, int n) {
  KRB_OP_BEGIN
  std::vector<float> v = h->e->last_logits();
  if (v.empty()) throw std::runtime_error("this rank produces no logits");
  if (n < int(v.size())) throw std::runtime_error("buffer too small");
  std::memcpy(out, v.data(), v.size() * 4);
  KRB_OP_END
}

KRB_EXPORT int krb_engine_final_hidden(krb_engine *h, float *out, size_t n) {
  KRB_OP_BEGIN
  const krb::ModelCfg &c = h->e->cfg();
  const size_t need = size_t(c.seq) * c.H;
  if (n < need) throw std::runtime_error("buffer too small");
  if (h->e->rank() != 0 && !h->e->microdag())
    throw std::runtime_error("only rank 0 holds the final hidden state");
  KRB_CUDA(cudaSetDevice(h->e->device()));
  KRB_CUDA(cudaStreamSynchronize(h->e->stream()));
  KRB_CUDA(cudaMemcpy(out, h->e->hidden_ptr(), need * 4, cudaMemcpyDeviceToHost));
  KRB_OP_END
}

KRB_EXPORT int krb_engine_final_x(krb_engine *h, uint16_t *out, size_t n) {
  KRB_OP_BEGIN
  const krb::ModelCfg &c = h->e->cfg();
  const size_t need = size_t(c.seq) * c.H;
  if (n < need) throw std::runtime_error("buffer too small");
  if (h->e->rank() != 0 && !h->e->microdag())
    throw std::runtime_error("only rank 0 holds the final normed rows");
  KRB_CUDA(cudaSetDevice(h->e->device()));
  KRB_CUDA(cudaStreamSynchronize(h->e->stream()));
  KRB_CUDA(cudaMemcpy(out, h->e->final_x_ptr(), need * 2, cudaMemcpyDeviceToHost));
  KRB_OP_END
}

KRB_EXPORT int krb_engine_info(krb_engine *h, char *out, size_t cap) {
  try {
    const krb::ModelCfg &c = h->e->cfg();
    std::ostringstream os;
    os << "{\"H\":" << c.H << ",\"I\":" << c.I << ",\"L\":" << c.L << ",\"HQ\":" << c.HQ
       << ",\"HKV\":" << c.HKV << ",\"D\":" << c.D << ",\"V\":" << c.V << ",\"seq\":" << c.seq
       << ",\"world\":" << h->e->world() << ",\"rank\":" << h->e->rank()
       << ",\"lm_rows\":" << h->e->lm_rows() << ",\"split\":" << (h->e->mode().split ? "true" : "false")
       << ",\"device\":" << h->e->device() << ",\"launches_per_run\":" << h->e->launches()
       << ",\"graph\":" << (h->e->mode().graph ? "true" : "false") << ",\"relay\":\""
       << h->e->relay_kind() << "\"}";
    return write_out(os.str(), out, cap);
  } catch (const std::exception &e) {
    return write_error(e.what(), out, cap);
  }
}

KRB_EXPORT int krb_engine_layer_dump(krb_engine *h, int on) {
  KRB_OP_BEGIN
  h->e->set_layer_dump(on != 0);
  KRB_OP_END
}

KRB_EXPORT int krb_engine_layer_hidden(krb_engine *h, int layer, float *out, size_t n) {
  KRB_OP_BEGIN
  std::vector<float> v = h->e->layer_hidden(layer);
  if (n < v.size()) throw std::runtime_error("buffer too small");
  std::memcpy(out, v.data(), v.size() * 4);
  KRB_OP_END
}

KRB_EXPORT int krb_engine_relay_trace(krb_engine *h, unsigned long long *out, size_t n,
                                      size_t *written) {
  KRB_OP_BEGIN
  std::vector<unsigned long long> v = h->e->relay_trace();
  if (n < v.size()) throw std::runtime_error("buffer too small");
  if (!v.empty()) std::memcpy(out, v.data(), v.size() * 8);
  if (written) *written = v.size();
  KRB_OP_END
}
