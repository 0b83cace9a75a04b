// Generic schedule executor behind kr_plan_run.
//
// Input: the reference scheduler's schedule.json (python/kernrelay/_vendor/scheduler/
// export.py): nodes {id, op, engine, rows, cols, k, n, dim0, tiles, split, iters, blocks,
// preds}, per-engine task streams {node, tile, wait, publish, in_row_off, in_rows,
// out_row_off, n_off, n_tiles, out_col_off, out_cols} and nranks.  Semantics follow
// exec/exec_main.cpp: ParseSchedule (:160-241), AllocateNode / UploadInputs (:434-540),
// PreparePlans (:542-704), EnqueueAll (:837-886), the graph modes (:948-1279),
// ChecksumAll (:1292-1311) and the result JSON (:1466-1479).
//
// B200 layout: one process, one host thread per rank, one CUDA stream per engine name
// (aicore / aic / aiv / aicpu / hccl — the names only label queues here; every queue runs
// on the same SMs), one device arena per rank holding every node buffer, inputs generated
// on the device from the reference's deterministic hash, cross-stream edges as CUDA
// events, collectives through NCCL.  Matmul B operands are stored K-major (transposed once
// at setup) for the tcgen05 GEMM.  Modes: direct (per-run enqueue), graph (the whole
// multi-stream schedule captured as ONE CUDA graph per rank — the reference's ACL graph
// mode only takes single-stream schedules), graph_per_stream (one graph per engine stream,
// cross-stream edges as external event nodes, launched in stream topological order) and
// graph_segment (graphs cut at every wait / publish, host events between them).
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "json_min.hpp"
#include "plan.h"
#include "plan_ops.h"
#include "ptx.cuh"

namespace krb {
namespace plan {

namespace {

using Clock = std::chrono::steady_clock;
using Key = std::pair<std::string, int>;

constexpr int kEngines = 5;
const char *const kEngineNames[kEngines] = {"aicore", "aic", "aiv", "aicpu", "hccl"};
constexpr size_t kChecksumElems = 8192;  // exec_main.cpp:1298
constexpr float kLayerNormEps = 1e-5f;   // op_impl.cpp:251

// exec_main.cpp:91-99
int engine_index(const std::string &e) {
  if (e == "aicore" || e == "compute") return 0;
  if (e == "aic") return 1;
  if (e == "aiv") return 2;
  if (e == "aicpu") return 3;
  if (e == "hccl") return 4;
  throw std::runtime_error("unknown engine " + e);
}

enum class Op {
  MatMul, Add, Gelu, Softmax, LayerNorm, Cast, TopK, Sort, Embedding,
  AllReduce, AllGather, ReduceScatter,
  CustomAivScale, CustomAicMac, CustomMixScale, CustomAicpuScale
};

// op_impl.cpp:59-76
Op parse_op(const std::string &name) {
  static const std::map<std::string, Op> ops = {
      {"matmul", Op::MatMul},       {"add", Op::Add},
      {"gelu", Op::Gelu},           {"softmax", Op::Softmax},
      {"layernorm", Op::LayerNorm}, {"cast", Op::Cast},
      {"topk", Op::TopK},           {"sort", Op::Sort},
      {"embedding", Op::Embedding}, {"allreduce", Op::AllReduce},
      {"allgather", Op::AllGather}, {"reducescatter", Op::ReduceScatter},
      {"custom_aiv_scale", Op::CustomAivScale},
      {"custom_aic_mac", Op::CustomAicMac},
      {"custom_mix_scale", Op::CustomMixScale},
      {"custom_aicpu_scale", Op::CustomAicpuScale}};
  auto it = ops.find(name);
  if (it == ops.end()) throw std::runtime_error("unknown op: " + name);
  return it->second;
}

bool is_comm(Op k) { return k == Op::AllReduce || k == Op::AllGather || k == Op::ReduceScatter; }

struct Node {
  std::string id;
  Op op = Op::Add;
  std::string engine = "aiv";
  int64_t rows = 0, cols = 0, k = 0, n = 0, dim0 = 0;
  int tiles = 1;
  bool split = false;
  uint32_t iters = 1, blocks = 1;
  std::vector<std::string> preds;
};

struct Task {
  std::string node;
  int tile = 0;
  std::vector<Key> waits;
  bool publish = false;
  Key key() const { return {node, tile}; }
};

struct Geom {
  int64_t in_row_off = 0, in_rows = 0, out_row_off = 0;
  int64_t n_off = 0, n_tile = 0, out_col_off = 0, out_cols = 0;
};

struct Lane {
  int engine = 0;
  std::vector<Task> tasks;
};

struct Doc {
  std::string dag, group;
  uint32_t nranks = 1;
  std::vector<Node> nodes;
  std::map<std::string, size_t> index;
  std::vector<Lane> lanes;  // non-empty lanes in engine order
  std::map<Key, Geom> geom;

  const Node &node(const std::string &id) const {
    auto it = index.find(id);
    if (it == index.end()) throw std::runtime_error("unknown node " + id);
    return nodes[it->second];
  }
  const Geom *geo(const Key &k) const {
    auto it = geom.find(k);
    return it == geom.end() ? nullptr : &it->second;
  }
};

int64_t rows_per_tile(const Node &n) { return n.split ? n.rows / n.tiles : n.rows; }
int tile_count(const Node &n) { return n.split ? n.tiles : 1; }

// exec_main.cpp:395-406: declared rows are input (send) rows
int64_t out_rows_of(const Node &n, uint32_t nranks) {
  switch (n.op) {
    case Op::AllGather: return int64_t(nranks) * n.rows;
    case Op::ReduceScatter: return n.rows / int64_t(nranks);
    default: return n.rows;
  }
}

// exec_main.cpp:420-432
size_t out_bytes_of(const Node &n, uint32_t nranks) {
  const size_t rows = size_t(n.rows), cols = size_t(n.cols);
  switch (n.op) {
    case Op::Cast: return rows * cols * 4;
    case Op::TopK: return rows * size_t(n.k) * 2 + rows * size_t(n.k) * 8;
    case Op::Sort: return rows * cols * 2 + rows * cols * 8;
    case Op::AllGather: return size_t(nranks) * rows * cols * 2;
    default: return rows * cols * 2;
  }
}

// element type of the checksummed output: fp32 for cast, fp16 otherwise
bool out_is_f32(const Node &n) { return n.op == Op::Cast; }

// exec_main.cpp:491-496 (FNV-1a of the node id, plus the rank)
uint32_t node_seed(const std::string &id, uint32_t rank) {
  uint32_t h = 2166136261u;
  for (char c : id) h = (h ^ uint8_t(c)) * 16777619u;
  return h + rank * 7919u;
}

int64_t num(const json::Value &v, const char *k, double d = 0) {
  return int64_t(v.number_or(k, d));
}

Doc parse(const json::Value &root) {
  Doc doc;
  doc.dag = root.string_or("dag", "");
  doc.group = root.string_or("group", "");
  doc.nranks = uint32_t(std::max<int64_t>(1, num(root, "nranks", 1)));
  for (const auto &n : root.at("nodes").arr) {
    Node s;
    s.id = n.at("id").str;
    s.op = parse_op(n.at("op").str);
    s.engine = n.string_or("engine", "aiv");
    s.rows = num(n, "rows");
    s.cols = num(n, "cols");
    s.k = num(n, "k");
    s.n = num(n, "n");
    s.dim0 = num(n, "dim0");
    s.tiles = int(num(n, "tiles", 1));
    s.split = n.bool_or("split", false);
    s.iters = uint32_t(num(n, "iters", 1));
    s.blocks = uint32_t(num(n, "blocks", 1));
    if (n.has("preds"))
      for (const auto &p : n.at("preds").arr) s.preds.push_back(p.str);
    if (doc.index.count(s.id)) throw std::runtime_error("duplicate node id " + s.id);
    doc.index[s.id] = doc.nodes.size();
    doc.nodes.push_back(s);
  }
  std::map<int, Lane> lanes;
  for (const auto &kv : root.at("streams").obj) {
    const int e = engine_index(kv.first);
    if (lanes.count(e))  // "compute" and "aicore" name the same lane (exec_main.cpp:261-266)
      throw std::runtime_error(std::string("duplicate engine stream ") + kEngineNames[e]);
    Lane lane;
    lane.engine = e;
    for (const auto &t : kv.second.arr) {
      Task task;
      task.node = t.at("node").str;
      task.tile = int(num(t, "tile", 0));
      task.publish = t.bool_or("publish", false);
      if (t.has("wait"))
        for (const auto &w : t.at("wait").arr)
          task.waits.emplace_back(w.arr.at(0).str, int(w.arr.at(1).num));
      if (t.has("in_row_off") && t.has("in_rows")) {
        Geom g;
        g.in_row_off = num(t, "in_row_off");
        g.in_rows = num(t, "in_rows");
        g.out_row_off = t.has("out_row_off") ? num(t, "out_row_off") : g.in_row_off;
        g.n_off = num(t, "n_off");
        g.n_tile = num(t, "n_tiles");
        g.out_col_off = t.has("out_col_off") ? num(t, "out_col_off") : g.n_off;
        g.out_cols = t.has("out_cols") ? num(t, "out_cols") : g.n_tile;
        if (doc.geom.count(task.key()))
          throw std::runtime_error("duplicate task for node " + task.node + " tile " +
                                   std::to_string(task.tile));
        doc.geom[task.key()] = g;
      }
      lane.tasks.push_back(task);
    }
    lanes[e] = std::move(lane);
  }
  for (auto &kv : lanes)
    if (!kv.second.tasks.empty()) doc.lanes.push_back(std::move(kv.second));
  return doc;
}

std::string key_str(const Key &k) { return k.first + "#" + std::to_string(k.second); }

// Task geometry of (node, tile): the schedule's explicit rows, else the stride rule
// (exec_main.cpp:565-567).
Geom task_geom(const Doc &doc, const Node &node, int t) {
  const Geom *g = doc.geo({node.id, t});
  if (g) return *g;
  Geom d;
  d.in_row_off = int64_t(t) * rows_per_tile(node);
  d.in_rows = rows_per_tile(node);
  d.out_row_off = d.in_row_off;
  return d;
}

// Every check the reference makes while preparing and enqueueing, done before any device
// work so a bad schedule fails fast (and without a GPU).
void validate(const Doc &doc) {
  std::map<Key, int> lane_of;
  std::set<Key> published;
  for (size_t l = 0; l < doc.lanes.size(); ++l) {
    for (const auto &t : doc.lanes[l].tasks) {
      auto it = doc.index.find(t.node);
      if (it == doc.index.end() || t.tile < 0 || t.tile >= tile_count(doc.nodes[it->second]))
        throw std::runtime_error("missing plan for task " + key_str(t.key()));
      if (lane_of.count(t.key()))
        throw std::runtime_error("duplicate task for node " + t.node + " tile " +
                                 std::to_string(t.tile));
      lane_of[t.key()] = int(l);
      if (t.publish) published.insert(t.key());
    }
  }
  for (const auto &lane : doc.lanes)
    for (const auto &t : lane.tasks)
      for (const auto &w : t.waits)
        if (!published.count(w)) throw std::runtime_error("wait on unpublished flag " + key_str(w));
  // wait cycle: Kahn over (lane FIFO + wait) edges
  {
    std::map<Key, std::vector<Key>> succ;
    std::map<Key, int> indeg;
    for (const auto &lane : doc.lanes) {
      for (size_t i = 0; i < lane.tasks.size(); ++i) {
        const Key k = lane.tasks[i].key();
        indeg[k] += 0;
        if (i > 0) {
          succ[lane.tasks[i - 1].key()].push_back(k);
          ++indeg[k];
        }
        for (const auto &w : lane.tasks[i].waits) {
          succ[w].push_back(k);
          ++indeg[k];
        }
      }
    }
    std::vector<Key> ready;
    for (const auto &kv : indeg)
      if (kv.second == 0) ready.push_back(kv.first);
    size_t done = 0;
    while (!ready.empty()) {
      const Key k = ready.back();
      ready.pop_back();
      ++done;
      for (const auto &s : succ[k])
        if (--indeg[s] == 0) ready.push_back(s);
    }
    if (done != indeg.size()) throw std::runtime_error("schedule contains wait cycle");
  }
  // node shapes and per-task geometry (exec_main.cpp:555-605, plus the full output extent)
  for (const auto &node : doc.nodes) {
    const std::string nm = node.id;
    if (node.rows <= 0 || node.cols <= 0) throw std::runtime_error("node " + nm + ": empty shape");
    if (node.tiles < 1 || (node.split && node.rows % node.tiles != 0))
      throw std::runtime_error("node " + nm + ": rows not divisible by tiles");
    for (const auto &p : node.preds) (void)doc.node(p);
    if (node.op == Op::MatMul) {
      if (node.k <= 0 || node.n <= 0) throw std::runtime_error("matmul " + nm + ": empty K or N");
      if (node.k % 8 || node.n % 8)
        throw std::runtime_error("matmul " + nm + ": K and N must be multiples of 8 on B200");
      if (node.cols != node.n) throw std::runtime_error("matmul " + nm + ": cols must equal n");
    }
    if (node.op == Op::TopK && (node.k <= 0 || node.k > node.cols))
      throw std::runtime_error("topk " + nm + ": k out of range");
    if ((node.op == Op::TopK || node.op == Op::Sort) && node.cols > kMaxSortCols)
      throw std::runtime_error("node " + nm + ": sort/topk rows longer than 16384");
    if (node.op == Op::Embedding && node.dim0 <= 0)
      throw std::runtime_error("embedding " + nm + ": dim0 must be positive");
    if (node.op == Op::ReduceScatter && node.rows % doc.nranks)
      throw std::runtime_error("reducescatter " + nm + ": rows not divisible by nranks");
    for (int t = 0; t < tile_count(node); ++t) {
      const Geom g = task_geom(doc, node, t);
      const int64_t in_limit =
          node.preds.empty() ? node.rows : out_rows_of(doc.node(node.preds[0]), doc.nranks);
      if (g.in_row_off < 0 || g.in_rows <= 0 || g.in_row_off + g.in_rows > in_limit)
        throw std::runtime_error("task " + nm + "#" + std::to_string(t) + " input rows [" +
                                 std::to_string(g.in_row_off) + "," +
                                 std::to_string(g.in_row_off + g.in_rows) + ") exceed " +
                                 std::to_string(in_limit));
      int64_t out_extent = g.in_rows;
      if (node.op == Op::AllGather) out_extent = int64_t(doc.nranks) * g.in_rows;
      if (node.op == Op::ReduceScatter) {
        if (g.in_rows % doc.nranks)
          throw std::runtime_error("task " + nm + "#" + std::to_string(t) +
                                   ": rows not divisible by nranks");
        out_extent = g.in_rows / doc.nranks;
      }
      // rows of the output buffer this task writes: reduce-scatter writes rank r's block
      // at r * rows / nranks + out_row_off of a rows-high buffer (exec_main.cpp:628-631)
      const int64_t out_limit = out_rows_of(node, doc.nranks);
      const int64_t last_row =
          node.op == Op::ReduceScatter
              ? (int64_t(doc.nranks) - 1) * node.rows / doc.nranks + g.out_row_off + out_extent
              : g.out_row_off + out_extent;
      const int64_t buf_rows = node.op == Op::ReduceScatter ? node.rows : out_limit;
      if (g.out_row_off < 0 || g.out_row_off > out_limit || last_row > buf_rows)
        throw std::runtime_error("task " + nm + "#" + std::to_string(t) + " output rows exceed " +
                                 std::to_string(buf_rows));
      // node-owned buffers indexed by input rows: the allgather staging block and the
      // second add operand generated for the node
      const bool own_rows = node.op == Op::AllGather || (node.op == Op::Add && node.preds.size() < 2) ||
                            node.op == Op::Embedding;
      if (own_rows && g.in_row_off + g.in_rows > node.rows)
        throw std::runtime_error("task " + nm + "#" + std::to_string(t) + " input rows exceed " +
                                 std::to_string(node.rows));
      // every input read stays inside its producer's buffer
      const int64_t in_cols = node.op == Op::MatMul ? node.k : node.cols;
      const size_t need = size_t(g.in_row_off + g.in_rows) * size_t(in_cols) * 2;
      for (size_t p = 0; p < node.preds.size() && p < (node.op == Op::Add ? 2u : 1u); ++p)
        if (need > out_bytes_of(doc.node(node.preds[p]), doc.nranks))
          throw std::runtime_error("task " + nm + "#" + std::to_string(t) + " input rows exceed " +
                                   "the buffer of " + node.preds[p]);
      if (node.op == Op::MatMul && g.n_tile > 0) {
        if (g.n_off < 0 || g.n_off + g.n_tile > node.n || g.out_col_off < 0 ||
            g.out_col_off + g.n_tile > node.n)
          throw std::runtime_error("task " + nm + "#" + std::to_string(t) + " N tile out of range");
        if (g.n_off % 8 || g.n_tile % 8 || g.out_col_off % 8)
          throw std::runtime_error("task " + nm + "#" + std::to_string(t) +
                                   ": N tile offsets must be multiples of 8 on B200");
      }
    }
  }
}

// ------------------------------------------------------------------ per-rank runtime
struct NodeBuf {
  char *out = nullptr, *out2 = nullptr, *aux1 = nullptr, *aux2 = nullptr;
  char *owned_in = nullptr, *aux_recv = nullptr;
  size_t out_bytes = 0;
};

struct Segment {
  int lane = 0, start = 0, end = 0;
  std::vector<Key> waits, publishes;
  cudaGraphExec_t exec = nullptr;
};

struct RankCtx {
  uint32_t rank = 0, nranks = 1;
  int device = 0;
  cudaStream_t streams[kEngines] = {};
  cudaStream_t root = nullptr;
  ncclComm_t comm = nullptr;
  char *arena = nullptr;
  uint32_t *status = nullptr;
  std::map<std::string, NodeBuf> bufs;
  std::map<Key, std::function<void(cudaStream_t)>> plans;
  std::map<Key, cudaEvent_t> events;
  cudaEvent_t t_begin = nullptr, t_end[kEngines] = {}, fork = nullptr, join[kEngines] = {};
  cudaGraphExec_t graph = nullptr;
  cudaGraphExec_t lane_graphs[kEngines] = {};
  std::vector<Segment> segments;
  double last_device_us = 0;

  void release() {
    if (device < 0) return;
    cudaSetDevice(device);
    if (graph) cudaGraphExecDestroy(graph);
    for (auto &g : lane_graphs)
      if (g) cudaGraphExecDestroy(g);
    for (auto &s : segments)
      if (s.exec) cudaGraphExecDestroy(s.exec);
    for (auto &kv : events) cudaEventDestroy(kv.second);
    for (auto *e : {t_begin, fork})
      if (e) cudaEventDestroy(e);
    for (int i = 0; i < kEngines; ++i) {
      if (t_end[i]) cudaEventDestroy(t_end[i]);
      if (join[i]) cudaEventDestroy(join[i]);
      if (streams[i]) cudaStreamDestroy(streams[i]);
    }
    if (root) cudaStreamDestroy(root);
    if (arena) cudaFree(arena);
    device = -1;
  }
};

size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

// exec_main.cpp:434-489: the same buffers per node, carved from one arena
void allocate(RankCtx &ctx, const Doc &doc) {
  struct Req {
    std::string id;
    char *NodeBuf::*field;
    size_t bytes;
  };
  std::vector<Req> reqs;
  const uint32_t R = doc.nranks;
  for (const auto &node : doc.nodes) {
    const size_t rows = size_t(node.rows), cols = size_t(node.cols);
    NodeBuf &b = ctx.bufs[node.id];
    b.out_bytes = out_bytes_of(node, R);
    reqs.push_back({node.id, &NodeBuf::out, b.out_bytes});
    switch (node.op) {
      case Op::MatMul: reqs.push_back({node.id, &NodeBuf::aux1, size_t(node.k) * size_t(node.n) * 2}); break;
      case Op::Add:
        if (node.preds.size() < 2) reqs.push_back({node.id, &NodeBuf::aux2, rows * cols * 2});
        break;
      case Op::LayerNorm:
        reqs.push_back({node.id, &NodeBuf::aux1, cols * 2});
        reqs.push_back({node.id, &NodeBuf::aux2, cols * 2});
        break;
      case Op::TopK: reqs.push_back({node.id, &NodeBuf::out2, rows * size_t(node.k) * 8}); break;
      case Op::Sort: reqs.push_back({node.id, &NodeBuf::out2, rows * cols * 8}); break;
      case Op::Embedding:
        reqs.push_back({node.id, &NodeBuf::aux1, size_t(node.dim0) * cols * 2});
        reqs.push_back({node.id, &NodeBuf::aux2, rows * 8});
        break;
      case Op::AllGather: reqs.push_back({node.id, &NodeBuf::aux_recv, size_t(R) * rows * cols * 2}); break;
      default: break;
    }
    if (node.preds.empty() && node.op != Op::Embedding) {
      const size_t in_cols = node.op == Op::MatMul ? size_t(node.k) : cols;
      reqs.push_back({node.id, &NodeBuf::owned_in, rows * in_cols * 2});
    }
  }
  size_t total = 256;  // status word
  for (const auto &r : reqs) total += align_up(r.bytes);
  KRB_CUDA(cudaMalloc(&ctx.arena, total));
  KRB_CUDA(cudaMemsetAsync(ctx.arena, 0, total, ctx.root));
  ctx.status = reinterpret_cast<uint32_t *>(ctx.arena);
  size_t off = 256;
  for (const auto &r : reqs) {
    ctx.bufs[r.id].*(r.field) = ctx.arena + off;
    off += align_up(r.bytes);
  }
}

// exec_main.cpp:498-540, on the device
void generate_inputs(RankCtx &ctx, const Doc &doc) {
  cudaStream_t s = ctx.root;
  for (const auto &node : doc.nodes) {
    NodeBuf &b = ctx.bufs[node.id];
    const uint32_t seed = node_seed(node.id, ctx.rank);
    const uint64_t rows = uint64_t(node.rows), cols = uint64_t(node.cols);
    if (b.owned_in) {
      const uint64_t in_cols = node.op == Op::MatMul ? uint64_t(node.k) : cols;
      det_fill_f16(reinterpret_cast<__half *>(b.owned_in), rows * in_cols, seed + 1, s);
    }
    if (b.aux1) {
      if (node.op == Op::MatMul)
        det_fill_f16_t(reinterpret_cast<__half *>(b.aux1), node.k, node.n, seed + 2, s);
      else if (node.op == Op::Embedding)
        det_fill_f16(reinterpret_cast<__half *>(b.aux1), uint64_t(node.dim0) * cols, seed + 2, s);
      else
        det_fill_f16(reinterpret_cast<__half *>(b.aux1), cols, seed + 2, s);
    }
    if (b.aux2) {
      if (node.op == Op::LayerNorm)
        det_fill_f16(reinterpret_cast<__half *>(b.aux2), cols, seed + 3, s);
      else if (node.op == Op::Embedding)
        embedding_indices(reinterpret_cast<int64_t *>(b.aux2), node.rows, node.dim0, seed, s);
      else if (node.op == Op::Add)
        det_fill_f16(reinterpret_cast<__half *>(b.aux2), rows * cols, seed + 3, s);
    }
  }
}

void nccl_check(ncclResult_t r, const char *what) {
  if (r != ncclSuccess)
    throw std::runtime_error(std::string(what) + " failed: " + ncclGetErrorString(r));
}

// exec_main.cpp:542-704 + op_impl.cpp: one closure per (node, tile)
void prepare_plans(RankCtx &ctx, const Doc &doc) {
  const uint32_t R = doc.nranks;
  for (const auto &node : doc.nodes) {
    NodeBuf &b = ctx.bufs[node.id];
    const int64_t cols = node.cols;
    const int64_t in_cols = node.op == Op::MatMul ? node.k : cols;
    char *in_base = nullptr;
    if (!node.preds.empty())
      in_base = ctx.bufs[node.preds[0]].out;
    else if (node.op != Op::Embedding)
      in_base = b.owned_in;
    for (int t = 0; t < tile_count(node); ++t) {
      const Geom g = task_geom(doc, node, t);
      const int64_t rows = g.in_rows;
      char *in_tile = in_base ? in_base + g.in_row_off * in_cols * 2 : nullptr;
      char *out_tile = b.out + g.out_row_off * cols * 2;
      std::function<void(cudaStream_t)> fn;
      const auto *hin = reinterpret_cast<const __half *>(in_tile);
      auto *hout = reinterpret_cast<__half *>(out_tile);
      const uint64_t elems = uint64_t(rows) * uint64_t(cols);
      uint32_t *status = ctx.status;
      ncclComm_t comm = ctx.comm;
      switch (node.op) {
        case Op::MatMul: {
          const int64_t K = node.k;
          int64_t N = node.n, ldc = node.n;
          const __half *B = reinterpret_cast<const __half *>(b.aux1);
          __half *C = reinterpret_cast<__half *>(b.out) + g.out_row_off * node.n;
          if (g.n_tile > 0) {
            N = g.n_tile;
            B += g.n_off * K;  // K-major B: column block n_off.. is a row block
            C += g.out_col_off;
          }
          fn = [=](cudaStream_t s) {
            gemm_f16(hin, K, B, K, C, ldc, int(rows), int(N), int(K), 0, status, s);
          };
          break;
        }
        case Op::Add: {
          const __half *in2 =
              node.preds.size() > 1
                  ? reinterpret_cast<const __half *>(ctx.bufs[node.preds[1]].out) + g.in_row_off * cols
                  : reinterpret_cast<const __half *>(b.aux2) + g.in_row_off * cols;
          fn = [=](cudaStream_t s) { add_f16(hin, in2, hout, elems, s); };
          break;
        }
        case Op::Gelu: fn = [=](cudaStream_t s) { gelu_f16(hin, hout, elems, s); }; break;
        case Op::Softmax:
          fn = [=](cudaStream_t s) { softmax_rows_f16(hin, hout, rows, cols, s); };
          break;
        case Op::Cast: {
          float *o = reinterpret_cast<float *>(b.out) + g.out_row_off * cols;
          fn = [=](cudaStream_t s) { cast_f16_f32(hin, o, elems, s); };
          break;
        }
        case Op::LayerNorm: {
          const __half *w = reinterpret_cast<const __half *>(b.aux1);
          const __half *bb = reinterpret_cast<const __half *>(b.aux2);
          fn = [=](cudaStream_t s) { layernorm_rows_f16(hin, w, bb, hout, rows, cols, kLayerNormEps, s); };
          break;
        }
        case Op::TopK: {
          const int64_t k = node.k;
          __half *v = reinterpret_cast<__half *>(b.out) + g.out_row_off * k;
          int64_t *ix = reinterpret_cast<int64_t *>(b.out2) + g.out_row_off * k;
          fn = [=](cudaStream_t s) { topk_rows_f16(hin, rows, cols, k, v, ix, s); };
          break;
        }
        case Op::Sort: {
          int64_t *ix = reinterpret_cast<int64_t *>(b.out2) + g.out_row_off * cols;
          fn = [=](cudaStream_t s) { sort_rows_f16(hin, rows, cols, hout, ix, s); };
          break;
        }
        case Op::Embedding: {
          const __half *w = reinterpret_cast<const __half *>(b.aux1);
          const int64_t *ids = reinterpret_cast<const int64_t *>(b.aux2) + g.in_row_off;
          const int64_t V = node.dim0;
          fn = [=](cudaStream_t s) { embedding_f16(w, ids, hout, rows, cols, V, status, s); };
          break;
        }
        case Op::AllReduce:
          fn = [=](cudaStream_t s) {
            nccl_check(ncclAllReduce(in_tile, out_tile, elems, ncclHalf, ncclSum, comm, s),
                       "ncclAllReduce");
          };
          break;
        case Op::ReduceScatter: {
          // exec_main.cpp:628-631: this rank's block of the output, plus the task's offset
          char *recv = b.out + (size_t(ctx.rank) * size_t(node.rows) / R + size_t(g.out_row_off)) *
                                   size_t(cols) * 2;
          const uint64_t count = elems / R;
          fn = [=](cudaStream_t s) {
            nccl_check(ncclReduceScatter(in_tile, recv, count, ncclHalf, ncclSum, comm, s),
                       "ncclReduceScatter");
          };
          break;
        }
        case Op::AllGather: {
          // gather into a [rank][rows] staging block, then place rank r's rows at
          // out_row_off + r * rows (op_impl.cpp:460-480)
          char *raw = b.aux_recv + size_t(g.in_row_off) * R * size_t(cols) * 2;
          char *dst = b.out;
          const size_t tile_bytes = size_t(rows) * size_t(cols) * 2;
          const int64_t orow = g.out_row_off;
          fn = [=](cudaStream_t s) {
            nccl_check(ncclAllGather(in_tile, raw, elems, ncclHalf, comm, s), "ncclAllGather");
            for (uint32_t r = 0; r < R; ++r)
              KRB_CUDA(cudaMemcpyAsync(dst + (size_t(orow) + size_t(r) * size_t(rows)) * size_t(cols) * 2,
                                       raw + r * tile_bytes, tile_bytes, cudaMemcpyDeviceToDevice, s));
          };
          break;
        }
        case Op::CustomAivScale:
        case Op::CustomMixScale: {
          // custom_aiv.cpp:46-49 / custom_mix.cpp:35-38 (the MIX kernel's scalar side
          // writes nothing, so its result is the vector side's)
          const float k = node.op == Op::CustomAivScale ? 1.0009765625f : 1.001953125f;
          const uint32_t iters = node.iters;
          fn = [=](cudaStream_t s) { scale_f16(hin, hout, elems, k, iters, s); };
          break;
        }
        case Op::CustomAicMac:
        case Op::CustomAicpuScale: {
          if (elems > 0xFFFFFFFFull) throw std::runtime_error("custom op elems out of range");
          const bool aic = node.op == Op::CustomAicMac;
          const uint32_t blocks = aic ? std::max<uint32_t>(node.blocks, 1) : 1;
          const float acc0 = aic ? 0.03125f : 0.0f;
          const uint32_t iters = node.iters;
          fn = [=](cudaStream_t s) { mac_f16(hin, hout, uint32_t(elems), iters, blocks, acc0, s); };
          break;
        }
      }
      ctx.plans[{node.id, t}] = std::move(fn);
    }
  }
}

// exec_main.cpp:837-886: round-robin over the lanes, a task goes once all its waits have
// been recorded; cross-lane edges are events.
void enqueue_all(RankCtx &ctx, const Doc &doc) {
  std::vector<size_t> idx(doc.lanes.size(), 0);
  std::set<Key> recorded;
  size_t remaining = 0;
  for (const auto &l : doc.lanes) remaining += l.tasks.size();
  while (remaining > 0) {
    bool progress = false;
    for (size_t l = 0; l < doc.lanes.size(); ++l) {
      const Lane &lane = doc.lanes[l];
      if (idx[l] >= lane.tasks.size()) continue;
      const Task &task = lane.tasks[idx[l]];
      bool ready = true;
      for (const auto &w : task.waits)
        if (!recorded.count(w)) {
          ready = false;
          break;
        }
      if (!ready) continue;
      cudaStream_t s = ctx.streams[lane.engine];
      for (const auto &w : task.waits) KRB_CUDA(cudaStreamWaitEvent(s, ctx.events.at(w), 0));
      auto plan = ctx.plans.find(task.key());
      if (plan == ctx.plans.end()) throw std::runtime_error("missing plan for task " + key_str(task.key()));
      plan->second(s);
      if (task.publish) {
        KRB_CUDA(cudaEventRecord(ctx.events.at(task.key()), s));
        recorded.insert(task.key());
      }
      ++idx[l];
      --remaining;
      progress = true;
    }
    if (!progress) throw std::runtime_error("schedule contains wait cycle");
  }
}

// lanes in topological order of their cross-lane waits; empty if they form a cycle
std::vector<int> lane_topo_order(const Doc &doc) {
  std::map<std::string, int> node_lane;
  for (size_t l = 0; l < doc.lanes.size(); ++l)
    for (const auto &t : doc.lanes[l].tasks) node_lane[key_str(t.key())] = int(l);
  const int L = int(doc.lanes.size());
  std::vector<std::set<int>> succ(L);
  std::vector<int> indeg(L, 0);
  for (int l = 0; l < L; ++l)
    for (const auto &t : doc.lanes[l].tasks)
      for (const auto &w : t.waits) {
        const int src = node_lane.at(key_str(w));
        if (src != l && succ[src].insert(l).second) ++indeg[l];
      }
  std::vector<int> order;
  std::vector<bool> done(L, false);
  while (int(order.size()) < L) {
    bool progress = false;
    for (int l = 0; l < L; ++l) {
      if (done[l] || indeg[l] != 0) continue;
      order.push_back(l);
      done[l] = true;
      for (int v : succ[l]) --indeg[v];
      progress = true;
    }
    if (!progress) return {};
  }
  return order;
}

cudaGraphExec_t end_capture(cudaStream_t s) {
  cudaGraph_t g = nullptr;
  KRB_CUDA(cudaStreamEndCapture(s, &g));
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  KRB_CUDA(e);
  return exec;
}

void capture_whole(RankCtx &ctx, const Doc &doc) {
  KRB_CUDA(cudaStreamBeginCapture(ctx.root, cudaStreamCaptureModeThreadLocal));
  KRB_CUDA(cudaEventRecord(ctx.fork, ctx.root));
  for (const auto &l : doc.lanes) KRB_CUDA(cudaStreamWaitEvent(ctx.streams[l.engine], ctx.fork, 0));
  enqueue_all(ctx, doc);
  for (const auto &l : doc.lanes) {
    KRB_CUDA(cudaEventRecord(ctx.join[l.engine], ctx.streams[l.engine]));
    KRB_CUDA(cudaStreamWaitEvent(ctx.root, ctx.join[l.engine], 0));
  }
  ctx.graph = end_capture(ctx.root);
}

void capture_per_lane(RankCtx &ctx, const Doc &doc, const std::vector<int> &order) {
  for (int l : order) {
    const Lane &lane = doc.lanes[l];
    cudaStream_t s = ctx.streams[lane.engine];
    std::set<Key> own;
    for (const auto &t : lane.tasks) own.insert(t.key());
    KRB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    for (const auto &t : lane.tasks) {
      for (const auto &w : t.waits)
        if (!own.count(w)) KRB_CUDA(cudaStreamWaitEvent(s, ctx.events.at(w), cudaEventWaitExternal));
      ctx.plans.at(t.key())(s);
      if (t.publish) KRB_CUDA(cudaEventRecordWithFlags(ctx.events.at(t.key()), s, cudaEventRecordExternal));
    }
    ctx.lane_graphs[lane.engine] = end_capture(s);
  }
}

// exec_main.cpp:1150-1187: a segment starts at a waiting task and ends after a publishing one
std::vector<Segment> build_segments(const Doc &doc) {
  std::vector<Segment> out;
  for (size_t l = 0; l < doc.lanes.size(); ++l) {
    const auto &tasks = doc.lanes[l].tasks;
    int start = 0;
    auto close = [&](int end) {
      if (end <= start) return;
      Segment seg;
      seg.lane = int(l);
      seg.start = start;
      seg.end = end;
      seg.waits = tasks[start].waits;
      for (int i = start; i < end; ++i)
        if (tasks[i].publish) seg.publishes.push_back(tasks[i].key());
      out.push_back(seg);
    };
    for (int i = 0; i < int(tasks.size()); ++i) {
      if (i > start && !tasks[i].waits.empty()) {
        close(i);
        start = i;
      }
      if (tasks[i].publish) {
        close(i + 1);
        start = i + 1;
      }
    }
    close(int(tasks.size()));
  }
  return out;
}

void capture_segments(RankCtx &ctx, const Doc &doc) {
  ctx.segments = build_segments(doc);
  for (auto &seg : ctx.segments) {
    const Lane &lane = doc.lanes[seg.lane];
    cudaStream_t s = ctx.streams[lane.engine];
    KRB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    for (int i = seg.start; i < seg.end; ++i) ctx.plans.at(lane.tasks[i].key())(s);
    seg.exec = end_capture(s);
  }
}

void launch_segments(RankCtx &ctx, const Doc &doc) {
  std::set<Key> recorded;
  std::vector<bool> launched(ctx.segments.size(), false);
  size_t remaining = ctx.segments.size();
  while (remaining > 0) {
    bool progress = false;
    for (size_t i = 0; i < ctx.segments.size(); ++i) {
      if (launched[i]) continue;
      const Segment &seg = ctx.segments[i];
      bool ready = true;
      for (const auto &w : seg.waits)
        if (!recorded.count(w)) {
          ready = false;
          break;
        }
      if (!ready) continue;
      cudaStream_t s = ctx.streams[doc.lanes[seg.lane].engine];
      for (const auto &w : seg.waits) KRB_CUDA(cudaStreamWaitEvent(s, ctx.events.at(w), 0));
      KRB_CUDA(cudaGraphLaunch(seg.exec, s));
      for (const auto &p : seg.publishes) {
        KRB_CUDA(cudaEventRecord(ctx.events.at(p), s));
        recorded.insert(p);
      }
      launched[i] = true;
      --remaining;
      progress = true;
    }
    if (!progress) throw std::runtime_error("segment wait cycle");
  }
}

enum class Mode { Direct, Graph, GraphPerStream, GraphSegment };

Mode parse_mode(const std::string &m) {
  if (m == "direct") return Mode::Direct;
  if (m == "graph") return Mode::Graph;
  if (m == "graph_per_stream") return Mode::GraphPerStream;
  if (m == "graph_segment") return Mode::GraphSegment;
  throw std::runtime_error("unknown plan mode " + m);
}

// One run on one rank: bracket the lanes with timing events, enqueue or launch, wait.
void run_rank_once(RankCtx &ctx, const Doc &doc, Mode mode, const std::vector<int> &order) {
  KRB_CUDA(cudaSetDevice(ctx.device));
  KRB_CUDA(cudaEventRecord(ctx.t_begin, ctx.root));
  if (mode == Mode::Graph) {
    KRB_CUDA(cudaGraphLaunch(ctx.graph, ctx.root));
    KRB_CUDA(cudaEventRecord(ctx.t_end[0], ctx.root));
    KRB_CUDA(cudaStreamSynchronize(ctx.root));
    float ms = 0;
    KRB_CUDA(cudaEventElapsedTime(&ms, ctx.t_begin, ctx.t_end[0]));
    ctx.last_device_us = ms * 1e3;
    return;
  }
  for (const auto &l : doc.lanes) KRB_CUDA(cudaStreamWaitEvent(ctx.streams[l.engine], ctx.t_begin, 0));
  if (mode == Mode::Direct) {
    enqueue_all(ctx, doc);
  } else if (mode == Mode::GraphPerStream) {
    for (int l : order) {
      const int e = doc.lanes[l].engine;
      KRB_CUDA(cudaGraphLaunch(ctx.lane_graphs[e], ctx.streams[e]));
    }
  } else {
    launch_segments(ctx, doc);
  }
  for (const auto &l : doc.lanes) KRB_CUDA(cudaEventRecord(ctx.t_end[l.engine], ctx.streams[l.engine]));
  double dev_us = 0;
  for (const auto &l : doc.lanes) {
    KRB_CUDA(cudaStreamSynchronize(ctx.streams[l.engine]));
    float ms = 0;
    KRB_CUDA(cudaEventElapsedTime(&ms, ctx.t_begin, ctx.t_end[l.engine]));
    dev_us = std::max(dev_us, double(ms) * 1e3);
  }
  ctx.last_device_us = dev_us;
}

// One run over all ranks (one host thread per rank, exec_main.cpp:888-946); returns the
// host makespan and the device makespan in microseconds.
std::pair<double, double> run_all_once(std::vector<RankCtx> &ctxs, const Doc &doc, Mode mode,
                                       const std::vector<int> &order) {
  std::vector<double> end_us(ctxs.size(), 0.0);
  std::vector<std::string> errors(ctxs.size());
  const auto begin = Clock::now();
  auto body = [&](size_t r) {
    try {
      run_rank_once(ctxs[r], doc, mode, order);
      end_us[r] = std::chrono::duration<double, std::micro>(Clock::now() - begin).count();
    } catch (const std::exception &e) {
      errors[r] = e.what();
    }
  };
  if (ctxs.size() == 1) {
    body(0);
  } else {
    std::vector<std::thread> th;
    for (size_t r = 0; r < ctxs.size(); ++r) th.emplace_back(body, r);
    for (auto &t : th) t.join();
  }
  for (const auto &e : errors)
    if (!e.empty()) throw std::runtime_error("rank worker failed: " + e);
  double host = 0, dev = 0;
  for (size_t r = 0; r < ctxs.size(); ++r) {
    host = std::max(host, end_us[r]);
    dev = std::max(dev, ctxs[r].last_device_us);
  }
  return {host, dev};
}

double median(std::vector<double> v) {
  if (v.empty()) return 0.0;
  std::sort(v.begin(), v.end());
  const size_t m = v.size() / 2;
  return v.size() % 2 ? v[m] : 0.5 * (v[m - 1] + v[m]);
}

std::vector<int> parse_devices(const std::string &s, uint32_t nranks) {
  std::vector<int> devs;
  if (s.empty()) {
    for (uint32_t r = 0; r < nranks; ++r) devs.push_back(int(r));
    return devs;
  }
  size_t pos = 0;
  while (true) {
    const size_t comma = s.find(',', pos);
    const std::string tok = s.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
    if (tok.empty()) throw std::runtime_error("devices has empty entry");
    devs.push_back(std::stoi(tok));
    if (comma == std::string::npos) break;
    pos = comma + 1;
  }
  if (devs.size() != nranks)
    throw std::runtime_error("devices needs exactly " + std::to_string(nranks) + " devices");
  return devs;
}

std::string num_json(double v) {
  if (!std::isfinite(v)) return "null";
  std::ostringstream o;
  o.precision(10);
  o << v;
  return o.str();
}

std::string array_json(const std::vector<double> &v) {
  std::string s = "[";
  for (size_t i = 0; i < v.size(); ++i) s += (i ? "," : "") + num_json(v[i]);
  return s + "]";
}

// exec_main.cpp:1292-1311: the first 8192 output elements of every node on every rank.
// Cast outputs are summed as fp32 elements (reading them as fp16 halves, as the reference
// does, mixes mantissa bits into the sum and can give NaN).
std::map<std::string, double> checksums(std::vector<RankCtx> &ctxs, const Doc &doc) {
  std::map<std::string, double> out;
  for (auto &ctx : ctxs) {
    KRB_CUDA(cudaSetDevice(ctx.device));
    for (const auto &node : doc.nodes) {
      const NodeBuf &b = ctx.bufs.at(node.id);
      double sum = 0;
      if (out_is_f32(node)) {
        const size_t n = std::min<size_t>(b.out_bytes / 4, kChecksumElems);
        std::vector<float> h(n);
        KRB_CUDA(cudaMemcpy(h.data(), b.out, n * 4, cudaMemcpyDeviceToHost));
        for (float v : h) sum += v;
      } else {
        const size_t n = std::min<size_t>(b.out_bytes / 2, kChecksumElems);
        std::vector<__half> h(n);
        KRB_CUDA(cudaMemcpy(h.data(), b.out, n * 2, cudaMemcpyDeviceToHost));
        for (const __half &v : h) sum += double(__half2float(v));
      }
      out[node.id] += sum;
    }
  }
  return out;
}

struct Session {
  std::vector<RankCtx> ctxs;
  std::vector<ncclComm_t> comms;
  bool failed = false;
  ~Session() {
    for (auto &c : ctxs) c.release();
    for (auto c : comms) {
      if (!c) continue;
      if (failed)
        ncclCommAbort(c);
      else
        ncclCommDestroy(c);
    }
  }
};

Doc load(const std::string &path) {
  Doc doc = parse(json::parse_file(path));
  validate(doc);
  return doc;
}

}  // namespace

std::string check(const std::string &schedule_path) {
  const Doc doc = load(schedule_path);
  size_t tasks = 0, pubs = 0;
  std::string lanes = "[";
  for (size_t l = 0; l < doc.lanes.size(); ++l) {
    lanes += std::string(l ? "," : "") + "\"" + kEngineNames[doc.lanes[l].engine] + "\"";
    tasks += doc.lanes[l].tasks.size();
    for (const auto &t : doc.lanes[l].tasks) pubs += t.publish ? 1 : 0;
  }
  lanes += "]";
  std::ostringstream o;
  o << "{\"dag\":\"" << json::escape(doc.dag) << "\",\"group\":\"" << json::escape(doc.group)
    << "\",\"nranks\":" << doc.nranks << ",\"nodes\":" << doc.nodes.size() << ",\"tasks\":" << tasks
    << ",\"publishes\":" << pubs << ",\"lanes\":" << lanes
    << ",\"segments\":" << build_segments(doc).size()
    << ",\"lane_order_acyclic\":" << (lane_topo_order(doc).empty() ? "false" : "true") << "}";
  return o.str();
}

std::string run(const std::string &schedule_path, int iters, int warmup, const std::string &devices,
                const std::string &mode_name, const std::string &out_path) {
  const Mode mode = parse_mode(mode_name);
  const Doc doc = load(schedule_path);
  const uint32_t R = doc.nranks;
  const std::vector<int> devs = parse_devices(devices, R);
  std::vector<int> order = lane_topo_order(doc);
  if (mode == Mode::GraphPerStream && order.empty())
    throw std::runtime_error("graph_per_stream needs acyclic dependencies between engine streams");
  iters = std::max(iters, 1);
  warmup = std::max(warmup, 0);

  int ndev = 0;
  KRB_CUDA(cudaGetDeviceCount(&ndev));
  for (int d : devs)
    if (d < 0 || d >= ndev) throw std::runtime_error("device " + std::to_string(d) + " not present");

  Session ses;
  ses.ctxs.resize(R);
  bool has_comm = false;
  for (const auto &n : doc.nodes) has_comm |= is_comm(n.op);
  try {
    if (has_comm) {
      ses.comms.assign(R, nullptr);
      std::vector<int> d = devs;
      nccl_check(ncclCommInitAll(ses.comms.data(), int(R), d.data()), "ncclCommInitAll");
    }
    for (uint32_t r = 0; r < R; ++r) {
      RankCtx &ctx = ses.ctxs[r];
      ctx.rank = r;
      ctx.nranks = R;
      ctx.device = devs[r];
      ctx.comm = has_comm ? ses.comms[r] : nullptr;
      KRB_CUDA(cudaSetDevice(ctx.device));
      KRB_CUDA(cudaStreamCreateWithFlags(&ctx.root, cudaStreamNonBlocking));
      for (int e = 0; e < kEngines; ++e) {
        KRB_CUDA(cudaStreamCreateWithFlags(&ctx.streams[e], cudaStreamNonBlocking));
        KRB_CUDA(cudaEventCreate(&ctx.t_end[e]));
        KRB_CUDA(cudaEventCreateWithFlags(&ctx.join[e], cudaEventDisableTiming));
      }
      KRB_CUDA(cudaEventCreate(&ctx.t_begin));
      KRB_CUDA(cudaEventCreateWithFlags(&ctx.fork, cudaEventDisableTiming));
      for (const auto &l : doc.lanes)
        for (const auto &t : l.tasks)
          if (t.publish && !ctx.events.count(t.key())) {
            cudaEvent_t ev = nullptr;
            KRB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
            ctx.events[t.key()] = ev;
          }
      allocate(ctx, doc);
      generate_inputs(ctx, doc);
      prepare_plans(ctx, doc);
      KRB_CUDA(cudaStreamSynchronize(ctx.root));
    }
    // one direct run first: sets kernel attributes outside any capture
    run_all_once(ses.ctxs, doc, Mode::Direct, order);
    if (mode != Mode::Direct) {
      for (auto &ctx : ses.ctxs) {
        KRB_CUDA(cudaSetDevice(ctx.device));
        if (mode == Mode::Graph)
          capture_whole(ctx, doc);
        else if (mode == Mode::GraphPerStream)
          capture_per_lane(ctx, doc, order);
        else
          capture_segments(ctx, doc);
      }
    }
    for (int i = 0; i < warmup; ++i) run_all_once(ses.ctxs, doc, mode, order);
    std::vector<double> host_us, dev_us;
    for (int i = 0; i < iters; ++i) {
      const auto t = run_all_once(ses.ctxs, doc, mode, order);
      host_us.push_back(t.first);
      dev_us.push_back(t.second);
    }
    uint32_t status = 0;
    for (auto &ctx : ses.ctxs) {
      KRB_CUDA(cudaSetDevice(ctx.device));
      KRB_CUDA(cudaDeviceSynchronize());
      uint32_t s = 0;
      KRB_CUDA(cudaMemcpy(&s, ctx.status, 4, cudaMemcpyDeviceToHost));
      status |= s;
    }
    const auto sums = checksums(ses.ctxs, doc);
    double total = 0;
    for (const auto &kv : sums) total += kv.second;

    std::ostringstream o;
    o << "{\"dag\":\"" << json::escape(doc.dag) << "\",\"group\":\"" << json::escape(doc.group)
      << "\",\"nranks\":" << R << ",\"iters\":" << iters << ",\"warmup\":" << warmup
      << ",\"p50_us\":" << num_json(median(host_us)) << ",\"gate_timeouts\":0"
      << ",\"checksum\":" << num_json(total) << ",\"ok\":" << (status == 0 ? "true" : "false")
      << ",\"times_us\":" << array_json(host_us) << ",\"mode\":\"" << mode_name << "\""
      << ",\"device_p50_us\":" << num_json(median(dev_us))
      << ",\"device_times_us\":" << array_json(dev_us) << ",\"device_status\":" << status
      << ",\"devices\":[";
    for (uint32_t r = 0; r < R; ++r) o << (r ? "," : "") << devs[r];
    o << "],\"lanes\":[";
    for (size_t l = 0; l < doc.lanes.size(); ++l)
      o << (l ? "," : "") << "\"" << kEngineNames[doc.lanes[l].engine] << "\"";
    o << "],\"node_checksums\":{";
    bool first = true;
    for (const auto &kv : sums) {
      o << (first ? "" : ",") << "\"" << json::escape(kv.first) << "\":" << num_json(kv.second);
      first = false;
    }
    o << "}}";
    const std::string res = o.str();
    std::ofstream f(out_path);
    if (!f) throw std::runtime_error("cannot write " + out_path);
    f << res << "\n";
    return res;
  } catch (...) {
    ses.failed = true;
    throw;
  }
}

}  // namespace plan
}  // namespace krb
