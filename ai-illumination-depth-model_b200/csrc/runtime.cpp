// Runtime behind the C ABI: the depth model (createDepthModel / DepthModel,
// src/model/runner.ts:79-485), the stateless shading entry point
// (src/lighting/renderer.ts + shade.ts + composite.ts), the per-kernel entry
// points and the synthetic-workload helpers.
//
// Model life cycle: create() parses or synthesises the weights, plans and
// validates the arena exactly as the reference does, uploads the logical
// weights once and repacks them on the device into the kernels' layouts, and
// allocates ONE device arena sized for max_batch frames plus the bilateral
// guide and the depth ping-pong. forward() records the op list (40 launches)
// into a CUDA graph on first use for a given (n, pointers) and replays it;
// nothing is allocated per call.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <mutex>

#include "host.h"
#include "illumina.h"
#include "kernels.h"
#include "pdl.cuh"

using namespace illumina;

namespace illumina {
namespace {
thread_local std::string g_last_error;
}
void set_last_error(const std::string &msg) { g_last_error = msg; }
}  // namespace illumina

#define ILL_TRY try {
#define ILL_CATCH                                          \
  }                                                        \
  catch (const Error &e) {                                 \
    set_last_error(e.what());                              \
    return e.status;                                       \
  }                                                        \
  catch (const std::bad_alloc &) {                         \
    set_last_error("out of host memory");                  \
    return ILLUMINA_INVALID_ARG;                           \
  }                                                        \
  catch (const std::exception &e) {                        \
    set_last_error(e.what());                              \
    return ILLUMINA_INVALID_ARG;                           \
  }

namespace {

// Split-K workspace of the tensor-core kernels: a model holds 16 MiB of fp32
// partial tiles (the planners split K only when a launch's partials fit); a
// per-kernel entry point call takes 8 MiB.
constexpr size_t kSplitKBytes = 16u << 20;
constexpr size_t kSplitKOpBytes = 8u << 20;
// Largest batch whose forward uses programmatic dependent launch.
constexpr int kPdlMaxBatch = 16;

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw Error(ILLUMINA_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

bool is_device_ptr(const void *p) {
  if (!p) return false;
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// A captured forward is keyed by its shape; the caller's frame / disparity /
// depth_low pointers are re-targeted in place on replay.
struct GraphKey {
  int n, layout, mode, has_low;
  const void *hist, *tex;
  bool operator==(const GraphKey &o) const {
    return n == o.n && layout == o.layout && mode == o.mode && has_low == o.has_low && hist == o.hist &&
           tex == o.tex;
  }
};

// Graph nodes whose pointer arguments depend on the caller's buffers.
struct CaptureNodes {
  cudaGraphNode_t pre = nullptr, bil = nullptr, low = nullptr;
  int pre_nargs = 0, pre_frames_arg = 0;  // argument list of the node that reads the frames
};

struct GraphEntry {
  GraphKey key;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  CaptureNodes nodes;
  const void *frames = nullptr, *disp = nullptr, *low = nullptr;
};

struct OpWeights {
  const float *w = nullptr, *b = nullptr, *dw_w = nullptr, *dw_b = nullptr;
  float head_bias = 0.0f;
};

}  // namespace

struct illumina_model {
  Architecture arch;
  ArenaPlan plan;
  illumina_model_options opts{};
  int device = 0;
  int T = gpu::F32;
  size_t elt = 4;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_join = nullptr, ev_done = nullptr;
  // host-buffer forwards run in frame chunks: uploads on copy_in and
  // downloads on copy_out overlap the graph of the neighbouring chunks
  static constexpr int kMaxChunks = 16;
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t ev_in[kMaxChunks] = {}, ev_fwd[kMaxChunks] = {};
  cudaEvent_t ev_out = nullptr;
  std::vector<float> host_weights;  // logical blob (kept for debug / re-pack)
  float *d_weights_logical = nullptr;
  float *d_weights = nullptr;
  std::vector<OpWeights> opw;
  char *d_arena = nullptr;
  size_t arena_alloc = 0;
  std::vector<size_t> buf_off;
  float *d_luma = nullptr;
  float *d_scene = nullptr;
  float *d_tex[2] = {nullptr, nullptr};
  float *d_stage_in = nullptr, *d_stage_out = nullptr, *d_stage_low = nullptr;
  // illumina_forward_async: two slots of device staging (frames in, disparity
  // out, allocated on the first asynchronous call) used alternately, so one
  // call's upload and download overlap its neighbours' graphs
  float *d_async_in[2] = {nullptr, nullptr}, *d_async_out[2] = {nullptr, nullptr};
  cudaEvent_t ev_async_in[2] = {}, ev_async_graph[2] = {}, ev_async_out[2] = {};
  uint8_t *d_async_src[2] = {nullptr, nullptr};  // 8-bit sources too large for a slot's tail
  size_t d_async_src_bytes = 0;
  int async_slot = 0;
  // 8-bit source images of a host-buffer illumina_forward_source that do not
  // fit behind the planar frames in d_stage_in (allocated on first need)
  uint8_t *d_src = nullptr;
  size_t d_src_bytes = 0;
  size_t device_bytes = 0;
  int history_index = 0, last_written = 1;
  float exposure = 1, range_sigma = 0.12f, base_alpha = 0.35f, sensitivity = 3.0f;
  std::vector<GraphEntry> graphs;
  int launches_per_forward = 0;
  int engine = ILLUMINA_ENGINE_TENSOR;
  std::vector<gpu::TcWeights> tcw;   // per op (pw / dwpw / lateral)
  std::vector<size_t> tc_off;        // per op: byte offset into d_wimg
  uint8_t *d_wimg = nullptr;         // tensor-core weight images
  // Error word, set (plain store) by a kernel that gave up a bounded wait:
  // pinned host memory mapped into the device, so the host reads it after a
  // launch without a copy on the stream.
  volatile int *h_err = nullptr;
  int *d_err = nullptr;              // device address of h_err
  long long wait_cycles = 0;         // tensor kernels' pipeline wait limit (0: the kernels' default)
  float *d_splitk = nullptr;         // split-K partial tiles of the tensor dw->pw kernel
  int stem_fused_op = -1;            // conv op folded into the preprocess launch, or -1
  int head_fused_op = -1;            // head op folded into the preceding dw->pw launch, or -1
  bool stem_writes_input = true;     // the folded launch still writes the network input

  void *tensor(const std::string &name) {
    auto it = plan.assignment.find(name);
    if (it == plan.assignment.end()) throw Error(ILLUMINA_INVALID_ARG, "runner: " + name + " has no arena buffer");
    return d_arena + buf_off[it->second];
  }
  void clear_graphs() {
    for (auto &g : graphs) {
      cudaGraphExecDestroy(g.exec);
      cudaGraphDestroy(g.graph);
    }
    graphs.clear();
  }
  ~illumina_model();
};

illumina_model::~illumina_model() {
  if (device >= 0) cudaSetDevice(device);
  // asynchronous forwards may still read or write the staging buffers
  if (stream) cudaStreamSynchronize(stream);
  if (copy_in) cudaStreamSynchronize(copy_in);
  if (copy_out) cudaStreamSynchronize(copy_out);
  clear_graphs();
  cudaFree(d_weights_logical);
  cudaFree(d_weights);
  cudaFree(d_arena);
  cudaFree(d_luma);
  cudaFree(d_scene);
  cudaFree(d_tex[0]);
  cudaFree(d_tex[1]);
  cudaFree(d_stage_in);
  cudaFree(d_stage_out);
  cudaFree(d_stage_low);
  cudaFree(d_src);
  for (int k = 0; k < 2; k++) {
    cudaFree(d_async_in[k]);
    cudaFree(d_async_out[k]);
    cudaFree(d_async_src[k]);
    if (ev_async_in[k]) cudaEventDestroy(ev_async_in[k]);
    if (ev_async_graph[k]) cudaEventDestroy(ev_async_graph[k]);
    if (ev_async_out[k]) cudaEventDestroy(ev_async_out[k]);
  }
  cudaFree(d_wimg);
  if (h_err) cudaFreeHost((void *)h_err);
  cudaFree(d_splitk);
  if (ev_join) cudaEventDestroy(ev_join);
  if (ev_done) cudaEventDestroy(ev_done);
  for (int i = 0; i < kMaxChunks; i++) {
    if (ev_in[i]) cudaEventDestroy(ev_in[i]);
    if (ev_fwd[i]) cudaEventDestroy(ev_fwd[i]);
  }
  if (ev_out) cudaEventDestroy(ev_out);
  if (copy_in) cudaStreamDestroy(copy_in);
  if (copy_out) cudaStreamDestroy(copy_out);
  if (stream) cudaStreamDestroy(stream);
}

namespace {

template <typename F>
size_t write_json(const std::string &s, char *buf, size_t cap, size_t *needed, F) {
  if (needed) *needed = s.size() + 1;
  if (buf && cap > 0) {
    size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return s.size() + 1;
}

gpu::PreprocessParams preprocess_params(const illumina_model &m) {
  gpu::PreprocessParams p;
  for (int i = 0; i < 3; i++) {
    p.mean[i] = (float)m.arch.mean[i];
    p.std[i] = (float)m.arch.std[i];
    p.inv_std[i] = (float)(1.0 / m.arch.std[i]);
  }
  p.exposure = m.exposure;
  p.decode_srgb = m.opts.decode_srgb ? 1 : 0;
  return p;
}

// runner.ts:466-476: a tensor is stolen (not readable after the forward) when
// a later op writes the buffer it was assigned.
bool tensor_live_at_end(const illumina_model &m, const std::string &name) {
  auto as = m.plan.assignment.find(name);
  if (as == m.plan.assignment.end()) return false;
  int produced = -1;
  for (size_t i = 0; i < m.arch.ops.size(); i++)
    if (m.arch.ops[i].out == name) {
      produced = (int)i;
      break;
    }
  for (size_t i = 0; i < m.arch.ops.size(); i++) {
    if ((int)i <= produced) continue;
    auto o = m.plan.assignment.find(m.arch.ops[i].out);
    if (o != m.plan.assignment.end() && o->second == as->second) return false;
  }
  return true;
}

// Folds the stem into the preprocess launch when the preprocess output's only
// reader is the op right after it, a 3x3 stride-2 conv from 4 to 16 channels.
// The input tensor is then written only when it is readable after the forward
// (kept intermediates, or a buffer no later op reuses).
void plan_stem_fusion(illumina_model &m) {
  m.stem_fused_op = -1;
  const auto &ops = m.arch.ops;
  if (ops.size() < 2 || ops[0].kind != OpKind::Preprocess) return;
  const Op &c = ops[1];
  if (c.kind != OpKind::Conv || c.in != ops[0].out || c.k != 3 || c.stride != 2) return;
  if (m.arch.shape(c.in).c != 4 || m.arch.shape(c.out).c != 16) return;
  for (size_t i = 2; i < ops.size(); i++)
    for (const auto &t : op_inputs(ops[i]))
      if (t == ops[0].out) return;
  m.stem_fused_op = 1;
  m.stem_writes_input = m.opts.keep_intermediates != 0 || tensor_live_at_end(m, ops[0].out);
}

// Folds the head into the dw->pw op right before it when that op produces the
// head's input (tensor engine only; the op's output is still written, and
// tc_dw launches the head itself when its tiling cannot fold it).
void plan_head_fusion(illumina_model &m) {
  m.head_fused_op = -1;
  if (m.engine != ILLUMINA_ENGINE_TENSOR) return;
  const auto &ops = m.arch.ops;
  for (size_t i = 1; i < ops.size(); i++)
    if (ops[i].kind == OpKind::Head && ops[i - 1].kind == OpKind::Dwpw && ops[i].in == ops[i - 1].out) {
      m.head_fused_op = (int)i;
      return;
    }
}

// Enqueues the whole op list on m.stream. mode 0: independent frames -> disp;
// mode 1: streaming frame with history (n == 1).
// The node most recently added to the graph being captured on `st`.
cudaGraphNode_t last_captured_node(cudaStream_t st) {
  cudaStreamCaptureStatus status;
  const cudaGraphNode_t *deps = nullptr;
  size_t nd = 0;
  cuda_check(cudaStreamGetCaptureInfo(st, &status, nullptr, nullptr, &deps, &nd), "capture info");
  if (status != cudaStreamCaptureStatusActive || nd != 1 || !deps)
    throw Error(ILLUMINA_CUDA_ERROR, "graph capture: expected a single tail node");
  return deps[0];
}

// from_input: the network input is already in the arena (the preprocess
// output, e.g. from an activation bundle): preprocess is skipped and the stem
// runs as its own conv launch.
int enqueue_forward(illumina_model &m, int n, const float *frames, int layout, float *disp, float *low_out,
                    const float *history, float *out_tex, const std::vector<cudaEvent_t> *marks = nullptr,
                    CaptureNodes *nodes = nullptr, bool from_input = false) {
  const Architecture &a = m.arch;
  const int S = a.input_size;
  int launches = 0;
  cudaStream_t st = m.stream;
  // programmatic dependent launch for small batches (kernels overlap their
  // prologue with the predecessor's tail); restored when this forward is queued
  struct PdlScope {
    bool saved;
    explicit PdlScope(bool on) : saved(gpu::pdl_enabled()) { gpu::pdl_enabled() = on; }
    ~PdlScope() { gpu::pdl_enabled() = saved; }
  } pdl(n <= kPdlMaxBatch);
  for (size_t i = 0; i < a.ops.size(); i++) {
    const Op &op = a.ops[i];
    if (marks) cuda_check(cudaEventRecord((*marks)[i], st), "profile event");
    if (from_input && op.kind == OpKind::Preprocess) continue;
    if ((int)i == m.stem_fused_op && !from_input) continue;  // ran inside the preprocess launch
    const OpWeights &w = m.opw[i];
    switch (op.kind) {
      case OpKind::Preprocess:
        if (m.stem_fused_op >= 0) {
          // preprocess + stem in one kernel; the network input is written only
          // when it stays readable after the forward
          const Op &stem = a.ops[m.stem_fused_op];
          const OpWeights &sw = m.opw[m.stem_fused_op];
          cuda_check(gpu::stem_fused(m.T, frames, layout, n, S, preprocess_params(m), sw.w, sw.b, stem.act,
                                     m.tensor(stem.out), m.d_luma, m.d_scene,
                                     m.stem_writes_input ? m.tensor(op.out) : nullptr, st),
                     "preprocess+stem");
          if (nodes)
            nodes->pre = last_captured_node(st), nodes->pre_nargs = gpu::kStemArgCount,
            nodes->pre_frames_arg = gpu::kStemFramesArg;
        } else {
          cuda_check(gpu::preprocess(m.T, frames, layout, n, S, preprocess_params(m), m.tensor(op.out), m.d_luma,
                                     m.d_scene, st),
                     "preprocess");
          if (nodes)
            nodes->pre = last_captured_node(st), nodes->pre_nargs = gpu::kPreprocessArgCount,
            nodes->pre_frames_arg = gpu::kPreprocessFramesArg;
        }
        launches++;
        break;
      case OpKind::Conv: {
        const TensorShape &si = a.shape(op.in), &so = a.shape(op.out);
        cuda_check(gpu::conv(m.T, m.tensor(op.in), n, si.h, si.w, si.c, w.w, w.b, so.c, op.k, op.stride, op.act,
                             m.tensor(op.out), st),
                   op.name.c_str());
        launches++;
        break;
      }
      case OpKind::Pw:
      case OpKind::Dwpw:
      case OpKind::Lateral: {
        const TensorShape &so = a.shape(op.out);
        gpu::GemmOp g;
        g.n = n;
        g.wait_cycles = m.wait_cycles;
        g.dst = m.tensor(op.out);
        g.bias = w.b;
        g.w = w.w;
        g.N = so.c;
        g.act = op.act;
        g.OH = so.h, g.OW = so.w;
        g.M = (long)n * so.h * so.w;
        g.ws = m.d_splitk, g.ws_bytes = m.d_splitk ? kSplitKBytes : 0;  // split-K partials (pw, dw->pw)
        if (op.kind == OpKind::Lateral) {
          const TensorShape &ss = a.shape(op.skip);
          g.mode = 2;
          g.src = m.tensor(op.skip);
          g.coarse = m.tensor(op.coarse);
          g.K = ss.c;
        } else {
          const TensorShape &si = a.shape(op.in);
          g.src = m.tensor(op.in);
          g.K = si.c;
          g.res = op.residual.empty() ? nullptr : m.tensor(op.residual);
          if (op.kind == OpKind::Dwpw) {
            g.mode = 1;
            g.H = si.h, g.W = si.w;
            g.ks = op.k, g.stride = op.stride;
            g.mid_act = op.mid_act;
            g.dw_w = w.dw_w, g.dw_b = w.dw_b;
            if ((int)i + 1 == m.head_fused_op) {
              // the head that reads this op's output runs in its epilogue
              const OpWeights &hw = m.opw[i + 1];
              g.head_w = hw.w, g.head_b = hw.head_bias, g.head_dst = (float *)m.tensor(a.ops[i + 1].out);
            }
          } else {
            g.mode = 0;
          }
        }
        if (m.engine == ILLUMINA_ENGINE_TENSOR)
          cuda_check(gpu::tc_op(m.T, g, m.tcw[i], m.d_wimg + m.tc_off[i], m.d_err, st), op.name.c_str());
        else
          cuda_check(gpu::gemm(m.T, g, st), op.name.c_str());
        launches++;
        break;
      }
      case OpKind::Head: {
        const TensorShape &si = a.shape(op.in);
        long M = (long)n * si.h * si.w;
        float *low = (float *)m.tensor(op.out);
        if ((int)i != m.head_fused_op) {
          cuda_check(gpu::head(m.T, m.tensor(op.in), M, si.c, w.w, w.head_bias, low, nullptr, st), "head");
          launches++;
        }
        if (low_out) {
          cuda_check(cudaMemcpyAsync(low_out, low, sizeof(float) * M, cudaMemcpyDeviceToDevice, st), "depth_low copy");
          if (nodes) nodes->low = last_captured_node(st);
        }
        break;
      }
      case OpKind::BilateralUp: {
        const TensorShape &si = a.shape(op.in);
        gpu::BilateralParams bp{m.range_sigma, m.base_alpha, m.sensitivity};
        cuda_check(gpu::bilateral((const float *)m.tensor(op.in), n, si.h, si.w, m.d_luma, bp, disp, history,
                                  out_tex, st),
                   "bilateralUp");
        if (nodes) nodes->bil = last_captured_node(st);
        launches++;
        break;
      }
    }
  }
  if (marks) cuda_check(cudaEventRecord((*marks)[a.ops.size()], st), "profile event");
  return launches;
}

// Re-targets pointer argument `arg` of kernel node `node` in `e.exec`.
void patch_kernel_arg(GraphEntry &e, cudaGraphNode_t node, int nargs, int arg, const void *value) {
  cudaKernelNodeParams kp;
  cuda_check(cudaGraphKernelNodeGetParams(node, &kp), "kernel node params");
  std::vector<void *> args(kp.kernelParams, kp.kernelParams + nargs);
  const void *v = value;
  args[arg] = &v;
  kp.kernelParams = args.data();
  cuda_check(cudaGraphExecKernelNodeSetParams(e.exec, node, &kp), "retarget kernel node");
}

GraphEntry &graph_for(illumina_model &m, const GraphKey &key, const float *frames, float *disp, float *low,
                      const float *hist, float *tex) {
  for (auto &g : m.graphs) {
    if (!(g.key == key)) continue;
    if (g.frames != frames) {
      patch_kernel_arg(g, g.nodes.pre, g.nodes.pre_nargs, g.nodes.pre_frames_arg, frames);
      g.frames = frames;
    }
    if (g.disp != disp) {
      patch_kernel_arg(g, g.nodes.bil, gpu::kBilateralArgCount, gpu::kBilateralDstArg, disp);
      g.disp = disp;
    }
    if (low && g.low != low) {
      const TensorShape &ls = m.arch.shape("depth_low");
      size_t bytes = sizeof(float) * (size_t)key.n * ls.h * ls.w;
      cuda_check(cudaGraphExecMemcpyNodeSetParams1D(g.exec, g.nodes.low, low, m.tensor("depth_low"), bytes,
                                                    cudaMemcpyDeviceToDevice),
                 "retarget memcpy node");
      g.low = low;
    }
    return g;
  }
  if (m.graphs.size() >= 8) {
    cudaGraphExecDestroy(m.graphs.front().exec);
    cudaGraphDestroy(m.graphs.front().graph);
    m.graphs.erase(m.graphs.begin());
  }
  GraphEntry e;
  e.key = key;
  cuda_check(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal), "begin capture");
  int launches = 0;
  try {
    launches = enqueue_forward(m, key.n, frames, key.layout, disp, low, hist, tex, nullptr, &e.nodes);
  } catch (...) {
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(m.stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  cuda_check(cudaStreamEndCapture(m.stream, &e.graph), "end capture");
  cudaError_t err = cudaGraphInstantiate(&e.exec, e.graph, 0);
  if (err != cudaSuccess) {
    cudaGraphDestroy(e.graph);
    cuda_check(err, "graph instantiate");
  }
  e.frames = frames, e.disp = disp, e.low = low;
  m.launches_per_forward = launches;
  m.graphs.push_back(e);
  return m.graphs.back();
}

// Runs the hot path with caller pointers (host or device). Host pointers are
// staged through the model's device buffers and make the call synchronous.
// Chunk sizes of a host-buffer forward of n frames (returns the count, 1 =
// no chunking). Below 32 frames one launch; below 128 two halves; else chunks
// growing from 16 by 16 frames (16, 32, 48, ...; faster and capped for very
// large batches so there are at most kMaxChunks),
// then a last chunk of 16. The first upload and the last download are the
// only transfers nothing overlaps, so they are short; each later chunk's upload
// (43 us/frame at 55 GB/s) fits in the previous, smaller chunk's compute
// (53-77 us/frame), while chunks grow toward the batch sizes that run fastest.
int host_chunks(int n, int *sizes) {
  if (n < 32) return sizes[0] = n, 1;
  if (n < 128) return sizes[0] = (n + 1) / 2, sizes[1] = n - sizes[0], 2;
  constexpr int kMax = illumina_model::kMaxChunks;
  int k = 0, rem = n - 32, step = 32;
  sizes[k++] = 16;
  // largest growth step that still fits the chunk budget
  const int cap = std::max(128, ((rem + kMax - 3) / (kMax - 2) + 15) / 16 * 16);
  const int inc = std::max(16, (cap / 8 + 15) / 16 * 16);  // 16 up to batches of ~1800
  while (rem > 0) {
    int c = std::min(step, rem);
    if (rem - c < 16 || k == kMax - 2) c = rem;
    sizes[k++] = c, rem -= c;
    step = std::min(step + inc, cap);
  }
  sizes[k++] = 16;
  return k;
}

// Chunk sizes for a host-buffer forward whose frames upload ~3x faster than
// they compute (8-bit RGBA sources at the network resolution: ~15 us per
// 448 frame at 55 GB/s against ~50 us of compute): a first chunk of 8 (the
// only upload nothing overlaps), then chunks growing threefold while the
// uploads stay ahead of the compute, a chunk of 48 whose compute hides the
// largest chunk's download, and a last chunk of 8 (the only download nothing
// overlaps). Below 160 frames the planar-frame schedule. A pipeline model fed
// with the measured per-batch costs puts 8, 48, 144, 48, 8 within 1 % of the
// best five-chunk schedule at 256 frames.
int host_chunks_fast_upload(int n, int *sizes) {
  if (n < 160) return host_chunks(n, sizes);
  constexpr int kMax = illumina_model::kMaxChunks;
  int k = 0, rem = n - 8 - 48 - 8, step = 48;
  sizes[k++] = 8;
  while (rem > 0) {
    int c = std::min(step, rem);
    if (rem - c < 48 || k == kMax - 3) c = rem;
    sizes[k++] = c, rem -= c;
    step = std::min(3 * step, 1024);
  }
  sizes[k++] = 48;
  sizes[k++] = 8;
  return k;
}

// Reports a bounded device wait that gave up (the kernels set the model's
// error word and left the rest of their work undone, so the outputs of the
// forward that ran them are undefined): clears the word and throws TIMEOUT.
// `when` says which call's kernels the word covers.
void check_timeout(illumina_model &m, const char *when) {
  if (!m.h_err || *m.h_err == 0) return;
  cuda_check(cudaStreamSynchronize(m.stream), "synchronize");
  *m.h_err = 0;
  throw Error(ILLUMINA_TIMEOUT, std::string("a tensor-core kernel gave up a bounded wait (") + when +
                                    "); the outputs of that forward are undefined, the model is usable again");
}

void run_forward(illumina_model &m, const float *frames, int n, int layout, float *disp, float *low,
                 cudaStream_t caller, int mode) {
  if (n < 1 || n > m.opts.max_batch)
    throw Error(ILLUMINA_INVALID_ARG, "forward: batch " + std::to_string(n) + " outside [1, " +
                                          std::to_string(m.opts.max_batch) + "]");
  if (layout != ILLUMINA_FRAME_RGB_PLANAR && layout != ILLUMINA_FRAME_RGBA_INTERLEAVED)
    throw Error(ILLUMINA_INVALID_ARG, "forward: unknown frame layout " + std::to_string(layout));
  if (!frames) throw Error(ILLUMINA_INVALID_ARG, "forward: frames is null");
  cuda_check(cudaSetDevice(m.device), "cudaSetDevice");
  // a forward queued by an earlier call on device buffers may have given up
  check_timeout(m, "in an earlier call on this model");
  const int S = m.arch.input_size;
  const long frame_floats = (layout == ILLUMINA_FRAME_RGB_PLANAR ? 3L : 4L) * S * S;
  const long disp_floats = (long)S * S, low_floats = (long)(S / 2) * (S / 2);
  bool host_in = !is_device_ptr(frames);
  bool host_disp = disp && !is_device_ptr(disp);
  bool host_low = low && !is_device_ptr(low);
  bool sync = host_in || host_disp || host_low;

  cuda_check(cudaEventRecord(m.ev_join, caller), "event record");
  cuda_check(cudaStreamWaitEvent(m.stream, m.ev_join, 0), "stream wait");
  // the copy streams also wait for work queued on the model stream before
  // this call (an asynchronous forward may still read the staging buffers)
  cuda_check(cudaEventRecord(m.ev_join, m.stream), "event record");

  // Host buffers, whole batches: frame chunks, each uploaded on copy_in, run
  // through the (chunk-sized) graph on the model stream and downloaded on
  // copy_out, so PCIe traffic in both directions overlaps the neighbouring
  // chunks' compute. The results are the same as one launch per chunk:
  // frames are independent.
  int sizes[illumina_model::kMaxChunks], chunks = host_chunks(n, sizes);
  if (mode == 0 && (host_in || host_disp) && !low && chunks > 1) {
    cuda_check(cudaStreamWaitEvent(m.copy_in, m.ev_join, 0), "stream wait");
    cuda_check(cudaStreamWaitEvent(m.copy_out, m.ev_join, 0), "stream wait");
    // every upload first (a pageable download blocks the host until its chunk
    // is done; the uploads are queued by then), then graphs and downloads
    long starts[illumina_model::kMaxChunks];
    for (int k = 0, f = 0; k < chunks; f += sizes[k], k++) starts[k] = f;
    if (host_in)
      for (int k = 0; k < chunks; k++) {
        const long f0 = starts[k];
        const int nk = sizes[k];
        cuda_check(cudaMemcpyAsync(m.d_stage_in + f0 * frame_floats, frames + f0 * frame_floats,
                                   sizeof(float) * nk * frame_floats, cudaMemcpyHostToDevice, m.copy_in),
                   "frames H2D");
        cuda_check(cudaEventRecord(m.ev_in[k], m.copy_in), "event record");
      }
    for (int k = 0; k < chunks; k++) {
      const long f0 = starts[k];
      const int nk = sizes[k];
      const float *f_dev = (host_in ? m.d_stage_in : frames) + f0 * frame_floats;
      if (host_in) cuda_check(cudaStreamWaitEvent(m.stream, m.ev_in[k], 0), "stream wait");
      float *d_disp = (host_disp || !disp ? m.d_stage_out : disp) + f0 * disp_floats;
      GraphKey key{nk, layout, 0, 0, nullptr, nullptr};
      GraphEntry &g = graph_for(m, key, f_dev, d_disp, nullptr, nullptr, nullptr);
      cuda_check(cudaGraphLaunch(g.exec, m.stream), "graph launch");
      if (host_disp) {
        cuda_check(cudaEventRecord(m.ev_fwd[k], m.stream), "event record");
        cuda_check(cudaStreamWaitEvent(m.copy_out, m.ev_fwd[k], 0), "stream wait");
        cuda_check(cudaMemcpyAsync(disp + f0 * disp_floats, d_disp, sizeof(float) * nk * disp_floats,
                                   cudaMemcpyDeviceToHost, m.copy_out),
                   "disparity D2H");
      }
    }
    cuda_check(cudaEventRecord(m.ev_out, m.copy_out), "event record");
    cuda_check(cudaStreamWaitEvent(m.stream, m.ev_out, 0), "stream wait");
    cuda_check(cudaEventRecord(m.ev_done, m.stream), "event record");
    cuda_check(cudaStreamWaitEvent(caller, m.ev_done, 0), "caller wait");
    cuda_check(cudaStreamSynchronize(m.stream), "synchronize");
    check_timeout(m, "in this call");
    return;
  }

  const float *f_dev = frames;
  if (host_in) {
    size_t bytes = sizeof(float) * n * frame_floats;
    cuda_check(cudaMemcpyAsync(m.d_stage_in, frames, bytes, cudaMemcpyHostToDevice, m.stream), "frames H2D");
    f_dev = m.d_stage_in;
  }
  float *d_disp = host_disp ? m.d_stage_out : disp;
  float *d_low = host_low ? m.d_stage_low : low;
  if (!d_disp && mode == 0) d_disp = m.d_stage_out;

  const float *hist = nullptr;
  float *tex = nullptr;
  if (mode == 1) {
    m.last_written = 1 - m.history_index;
    hist = m.d_tex[m.history_index];
    tex = m.d_tex[1 - m.history_index];
  }
  GraphKey key{n, layout, mode, d_low ? 1 : 0, hist, tex};
  GraphEntry &g = graph_for(m, key, f_dev, d_disp, d_low, hist, tex);
  cuda_check(cudaGraphLaunch(g.exec, m.stream), "graph launch");

  if (host_disp)
    cuda_check(cudaMemcpyAsync(disp, m.d_stage_out, sizeof(float) * n * disp_floats, cudaMemcpyDeviceToHost, m.stream),
               "disparity D2H");
  if (host_low)
    cuda_check(cudaMemcpyAsync(low, m.d_stage_low, sizeof(float) * n * low_floats, cudaMemcpyDeviceToHost, m.stream),
               "depth_low D2H");
  cuda_check(cudaEventRecord(m.ev_done, m.stream), "event record");
  cuda_check(cudaStreamWaitEvent(caller, m.ev_done, 0), "caller wait");
  if (sync) {
    cuda_check(cudaStreamSynchronize(m.stream), "synchronize");
    check_timeout(m, "in this call");
  }
}

// The hot path from 8-bit RGBA source images (n x h x w x 4 bytes, host or
// device), the reference's frame path: a camera or canvas frame uploaded as an
// rgba8unorm texture and read by makePreprocess (src/model/kernels/io.ts:64-118)
// at uv * uv_scale + uv_offset. Each frame chunk's bytes are uploaded on
// copy_in, sampled to planar float frames on the model stream (the kernel of
// illumina_sample_source) and run through the chunk's graph; the disparity
// goes back on copy_out. A host source moves 4 bytes per source pixel over
// PCIe instead of the 12 of planar float frames at the network resolution.
void run_forward_source(illumina_model &m, const uint8_t *rgba8, int n, int w, int h, const float *uv_scale,
                        const float *uv_offset, int mirror, float *disp, cudaStream_t caller) {
  if (n < 1 || n > m.opts.max_batch)
    throw Error(ILLUMINA_INVALID_ARG, "forwardSource: batch " + std::to_string(n) + " outside [1, " +
                                          std::to_string(m.opts.max_batch) + "]");
  if (w < 1 || h < 1 || (long)w * h > (1L << 26))
    throw Error(ILLUMINA_INVALID_ARG, "forwardSource: source size " + std::to_string(w) + "x" + std::to_string(h) +
                                          " outside [1, 2^26] pixels");
  if (!rgba8) throw Error(ILLUMINA_INVALID_ARG, "forwardSource: rgba8 is null");
  if ((reinterpret_cast<uintptr_t>(rgba8) & 3) != 0)
    throw Error(ILLUMINA_INVALID_ARG, "forwardSource: rgba8 must be 4-byte aligned");
  cuda_check(cudaSetDevice(m.device), "cudaSetDevice");
  check_timeout(m, "in an earlier call on this model");
  const int S = m.arch.input_size;
  const long planar = 3L * S * S, disp_floats = (long)S * S;
  const size_t src_bytes = (size_t)w * h * 4;
  const float one[2] = {1.0f, 1.0f}, zero[2] = {0.0f, 0.0f};
  const float *us = uv_scale ? uv_scale : one, *uo = uv_offset ? uv_offset : zero;
  const bool host_in = !is_device_ptr(rgba8);
  const bool host_disp = disp && !is_device_ptr(disp);

  // a host source is staged behind the planar frames in d_stage_in (sized for
  // the interleaved RGBA layout: 4 floats per pixel) when it fits there
  const uint8_t *stage = nullptr;
  if (host_in) {
    const size_t tail = sizeof(float) * (size_t)m.opts.max_batch * (4L * S * S - planar);
    if (src_bytes * n <= tail) {
      stage = reinterpret_cast<uint8_t *>(m.d_stage_in + (size_t)m.opts.max_batch * planar);
    } else {
      if (m.d_src_bytes < src_bytes * n) {
        cuda_check(cudaStreamSynchronize(m.stream), "synchronize");
        cudaFree(m.d_src);
        m.d_src = nullptr, m.d_src_bytes = 0;
        cuda_check(cudaMalloc(&m.d_src, src_bytes * n), "cudaMalloc source staging");
        m.d_src_bytes = src_bytes * n;
      }
      stage = m.d_src;
    }
  }

  cuda_check(cudaEventRecord(m.ev_join, caller), "event record");
  cuda_check(cudaStreamWaitEvent(m.stream, m.ev_join, 0), "stream wait");
  // the copy streams also wait for work queued on the model stream before
  // this call (an asynchronous forward may still read the staging buffers)
  cuda_check(cudaEventRecord(m.ev_join, m.stream), "event record");
  cuda_check(cudaStreamWaitEvent(m.copy_in, m.ev_join, 0), "stream wait");
  cuda_check(cudaStreamWaitEvent(m.copy_out, m.ev_join, 0), "stream wait");
  int sizes[illumina_model::kMaxChunks], chunks = 1;
  if (host_in || host_disp)
    // sources of at most a third of a planar float frame's bytes upload fast
    chunks = host_in && src_bytes * 3 <= sizeof(float) * planar ? host_chunks_fast_upload(n, sizes)
                                                                : host_chunks(n, sizes);
  else
    sizes[0] = n;
  long starts[illumina_model::kMaxChunks];
  for (int k = 0, f = 0; k < chunks; f += sizes[k], k++) starts[k] = f;
  if (host_in)
    for (int k = 0; k < chunks; k++) {
      cuda_check(cudaMemcpyAsync(const_cast<uint8_t *>(stage) + starts[k] * src_bytes, rgba8 + starts[k] * src_bytes,
                                 src_bytes * sizes[k], cudaMemcpyHostToDevice, m.copy_in),
                 "source H2D");
      cuda_check(cudaEventRecord(m.ev_in[k], m.copy_in), "event record");
    }
  for (int k = 0; k < chunks; k++) {
    const long f0 = starts[k];
    const int nk = sizes[k];
    if (host_in) cuda_check(cudaStreamWaitEvent(m.stream, m.ev_in[k], 0), "stream wait");
    float *frames = m.d_stage_in + f0 * planar;
    cuda_check(gpu::sample_source((host_in ? stage : rgba8) + f0 * src_bytes, nk, w, h, us, uo, mirror ? 1 : 0, S,
                                  frames, m.stream),
               "sample_source");
    float *d_disp = (host_disp || !disp ? m.d_stage_out : disp) + f0 * disp_floats;
    GraphKey key{nk, ILLUMINA_FRAME_RGB_PLANAR, 0, 0, nullptr, nullptr};
    GraphEntry &g = graph_for(m, key, frames, d_disp, nullptr, nullptr, nullptr);
    cuda_check(cudaGraphLaunch(g.exec, m.stream), "graph launch");
    if (host_disp) {
      cuda_check(cudaEventRecord(m.ev_fwd[k], m.stream), "event record");
      cuda_check(cudaStreamWaitEvent(m.copy_out, m.ev_fwd[k], 0), "stream wait");
      cuda_check(cudaMemcpyAsync(disp + f0 * disp_floats, d_disp, sizeof(float) * nk * disp_floats,
                                 cudaMemcpyDeviceToHost, m.copy_out),
                 "disparity D2H");
    }
  }
  cuda_check(cudaEventRecord(m.ev_out, m.copy_out), "event record");
  cuda_check(cudaStreamWaitEvent(m.stream, m.ev_out, 0), "stream wait");
  cuda_check(cudaEventRecord(m.ev_done, m.stream), "event record");
  cuda_check(cudaStreamWaitEvent(caller, m.ev_done, 0), "caller wait");
  if (host_in || host_disp) {
    cuda_check(cudaStreamSynchronize(m.stream), "synchronize");
    check_timeout(m, "in this call");
  }
}

bool is_pinned_host(const void *p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// An asynchronous forward of pinned host buffers (the reference submits each
// frame without a fence, src/engine/frame.ts:1-19, and awaits readbacks
// asynchronously, src/main.ts:572-573):
// the frames go up on copy_in into one of two device slots, the whole batch
// runs as one graph on the model stream, the disparity comes down on copy_out;
// the call returns once that is queued. Consecutive calls alternate slots, so
// a call's upload and download overlap the neighbouring calls' graphs. The
// caller's stream is made to wait for the download (the upload does not wait
// for it); illumina_model_sync waits for everything queued.
// The 8-bit source of an asynchronous forward (illumina_forward_source_async).
struct AsyncSource {
  const uint8_t *rgba8;
  int w, h, mirror;
  const float *uv_scale, *uv_offset;
};

void run_forward_async(illumina_model &m, const float *frames, int n, int layout, float *disp, cudaStream_t caller,
                       const AsyncSource *src = nullptr) {
  const char *who = src ? "forwardSourceAsync" : "forwardAsync";
  if (n < 1 || n > m.opts.max_batch)
    throw Error(ILLUMINA_INVALID_ARG, std::string(who) + ": batch " + std::to_string(n) + " outside [1, " +
                                          std::to_string(m.opts.max_batch) + "]");
  if (layout != ILLUMINA_FRAME_RGB_PLANAR && layout != ILLUMINA_FRAME_RGBA_INTERLEAVED)
    throw Error(ILLUMINA_INVALID_ARG, std::string(who) + ": unknown frame layout " + std::to_string(layout));
  const void *in = src ? static_cast<const void *>(src->rgba8) : static_cast<const void *>(frames);
  if (!in || !disp) throw Error(ILLUMINA_INVALID_ARG, std::string(who) + ": input and disparity are required");
  size_t src_bytes = 0;
  if (src) {
    if (src->w < 1 || src->h < 1 || (long)src->w * src->h > (1L << 26))
      throw Error(ILLUMINA_INVALID_ARG, std::string(who) + ": source size outside [1, 2^26] pixels");
    if ((reinterpret_cast<uintptr_t>(src->rgba8) & 3) != 0)
      throw Error(ILLUMINA_INVALID_ARG, std::string(who) + ": rgba8 must be 4-byte aligned");
    src_bytes = (size_t)src->w * src->h * 4;
  }
  cuda_check(cudaSetDevice(m.device), "cudaSetDevice");
  if (!is_pinned_host(in) || !is_pinned_host(disp))
    throw Error(ILLUMINA_INVALID_ARG, std::string(who) +
                                          ": input and disparity must be pinned host memory (cudaHostAlloc / "
                                          "cudaHostRegister)");
  check_timeout(m, "in an earlier call on this model");
  const int S = m.arch.input_size;
  const long frame_floats = (layout == ILLUMINA_FRAME_RGB_PLANAR ? 3L : 4L) * S * S;
  const long planar = 3L * S * S, disp_floats = (long)S * S;
  if (!m.d_async_in[0]) {
    for (int k = 0; k < 2; k++) {
      cuda_check(cudaMalloc(&m.d_async_in[k], sizeof(float) * 4L * S * S * m.opts.max_batch), "cudaMalloc async");
      cuda_check(cudaMalloc(&m.d_async_out[k], sizeof(float) * disp_floats * m.opts.max_batch), "cudaMalloc async");
      cuda_check(cudaEventCreateWithFlags(&m.ev_async_in[k], cudaEventDisableTiming), "event create");
      cuda_check(cudaEventCreateWithFlags(&m.ev_async_graph[k], cudaEventDisableTiming), "event create");
      cuda_check(cudaEventCreateWithFlags(&m.ev_async_out[k], cudaEventDisableTiming), "event create");
    }
    m.device_bytes += 2 * sizeof(float) * (4L * S * S + disp_floats) * m.opts.max_batch;
  }
  // a source is staged behind the slot's planar frames when it fits there,
  // else in per-slot buffers grown on need (after everything queued is done)
  const size_t tail = sizeof(float) * (size_t)m.opts.max_batch * (4L * S * S - planar);
  if (src && src_bytes * n > tail && m.d_async_src_bytes < src_bytes * n) {
    cuda_check(cudaStreamSynchronize(m.stream), "synchronize");
    cuda_check(cudaStreamSynchronize(m.copy_in), "synchronize");
    cuda_check(cudaStreamSynchronize(m.copy_out), "synchronize");
    for (int k = 0; k < 2; k++) {
      cudaFree(m.d_async_src[k]);
      m.d_async_src[k] = nullptr;
    }
    m.d_async_src_bytes = 0;
    for (int k = 0; k < 2; k++) cuda_check(cudaMalloc(&m.d_async_src[k], src_bytes * n), "cudaMalloc async source");
    m.d_async_src_bytes = src_bytes * n;
  }
  const int k = m.async_slot;
  m.async_slot ^= 1;
  uint8_t *stage = nullptr;
  if (src)
    stage = src_bytes * n <= tail ? reinterpret_cast<uint8_t *>(m.d_async_in[k] + (size_t)m.opts.max_batch * planar)
                                  : m.d_async_src[k];
  // upload into slot k once the graph that last read it is done (the input
  // is host memory: nothing on the caller's stream precedes it, and waiting
  // on it would chain each call behind the previous call's download)
  cuda_check(cudaStreamWaitEvent(m.copy_in, m.ev_async_graph[k], 0), "stream wait");
  if (src)
    cuda_check(cudaMemcpyAsync(stage, src->rgba8, src_bytes * n, cudaMemcpyHostToDevice, m.copy_in), "source H2D");
  else
    cuda_check(cudaMemcpyAsync(m.d_async_in[k], frames, sizeof(float) * n * frame_floats, cudaMemcpyHostToDevice,
                               m.copy_in),
               "frames H2D");
  cuda_check(cudaEventRecord(m.ev_async_in[k], m.copy_in), "event record");
  // the graph once the upload is in and the download that last read slot k's output is done
  cuda_check(cudaStreamWaitEvent(m.stream, m.ev_async_in[k], 0), "stream wait");
  cuda_check(cudaStreamWaitEvent(m.stream, m.ev_async_out[k], 0), "stream wait");
  if (src) {
    const float one[2] = {1.0f, 1.0f}, zero[2] = {0.0f, 0.0f};
    cuda_check(gpu::sample_source(stage, n, src->w, src->h, src->uv_scale ? src->uv_scale : one,
                                  src->uv_offset ? src->uv_offset : zero, src->mirror ? 1 : 0, S, m.d_async_in[k],
                                  m.stream),
               "sample_source");
  }
  GraphKey key{n, layout, 0, 0, nullptr, nullptr};
  GraphEntry &g = graph_for(m, key, m.d_async_in[k], m.d_async_out[k], nullptr, nullptr, nullptr);
  cuda_check(cudaGraphLaunch(g.exec, m.stream), "graph launch");
  cuda_check(cudaEventRecord(m.ev_async_graph[k], m.stream), "event record");
  cuda_check(cudaStreamWaitEvent(m.copy_out, m.ev_async_graph[k], 0), "stream wait");
  cuda_check(cudaMemcpyAsync(disp, m.d_async_out[k], sizeof(float) * n * disp_floats, cudaMemcpyDeviceToHost,
                             m.copy_out),
             "disparity D2H");
  cuda_check(cudaEventRecord(m.ev_async_out[k], m.copy_out), "event record");
  cuda_check(cudaStreamWaitEvent(caller, m.ev_async_out[k], 0), "caller wait");
}

void build_model(illumina_model &m, const illumina_model_options &o) {
  m.opts = o;
  if (m.opts.max_batch < 1) throw Error(ILLUMINA_INVALID_ARG, "createDepthModel: max_batch must be >= 1");
  if (o.precision != ILLUMINA_PRECISION_F32 && o.precision != ILLUMINA_PRECISION_BF16)
    throw Error(ILLUMINA_INVALID_ARG, "createDepthModel: unknown precision " + std::to_string(o.precision));
  m.arch = build_architecture(o.input_size);
  m.T = o.precision == ILLUMINA_PRECISION_BF16 ? gpu::BF16 : gpu::F32;
  m.elt = m.T == gpu::BF16 ? 2 : 4;
  m.exposure = o.exposure;
  m.range_sigma = o.range_sigma;
  m.base_alpha = o.temporal_base;
  m.sensitivity = o.temporal_sensitivity;

  // --- weights (host) ---
  size_t count = weight_count(m.arch);
  if (o.weights && o.weights_count) {
    if (o.weights_count != count)
      throw Error(ILLUMINA_BAD_WEIGHTS, "weights: blob has " + std::to_string(o.weights_count) + " values, expected " +
                                            std::to_string(count));
    m.host_weights.assign(o.weights, o.weights + count);
  } else if (o.idm_bytes && o.idm_len) {
    m.host_weights = parse_weights(m.arch, (const uint8_t *)o.idm_bytes, o.idm_len);
  } else if (o.idm_path && o.idm_path[0]) {
    std::ifstream f(o.idm_path, std::ios::binary);
    if (!f) throw Error(ILLUMINA_BAD_WEIGHTS, std::string("weights: cannot open ") + o.idm_path);
    std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    m.host_weights = parse_weights(m.arch, bytes.data(), bytes.size());
  } else {
    m.host_weights = synthesize_weights(m.arch, o.synth_seed);
  }

  // --- arena plan (runner.ts:190-192) ---
  std::vector<std::string> exclude = {"depth"};
  m.plan = plan_arena(m.arch, exclude, o.keep_intermediates != 0);
  validate_arena(m.arch, m.plan, exclude);
  plan_stem_fusion(m);

  // --- device ---
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    throw Error(ILLUMINA_NO_DEVICE, "createDepthModel: no CUDA device");
  }
  if (o.device < 0 || o.device >= ndev)
    throw Error(ILLUMINA_INVALID_ARG, "createDepthModel: device " + std::to_string(o.device) + " out of range");
  m.device = o.device;
  cuda_check(cudaSetDevice(m.device), "cudaSetDevice");
  cuda_check(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking), "stream create");
  cuda_check(cudaEventCreateWithFlags(&m.ev_join, cudaEventDisableTiming), "event create");
  cuda_check(cudaEventCreateWithFlags(&m.ev_done, cudaEventDisableTiming), "event create");
  cuda_check(cudaStreamCreateWithFlags(&m.copy_in, cudaStreamNonBlocking), "stream create");
  cuda_check(cudaStreamCreateWithFlags(&m.copy_out, cudaStreamNonBlocking), "stream create");
  for (int i = 0; i < illumina_model::kMaxChunks; i++) {
    cuda_check(cudaEventCreateWithFlags(&m.ev_in[i], cudaEventDisableTiming), "event create");
    cuda_check(cudaEventCreateWithFlags(&m.ev_fwd[i], cudaEventDisableTiming), "event create");
  }
  cuda_check(cudaEventCreateWithFlags(&m.ev_out, cudaEventDisableTiming), "event create");

  // Upload the logical blob, then repack per op on the device.
  cuda_check(cudaMalloc(&m.d_weights_logical, count * 4), "cudaMalloc weights");
  cuda_check(cudaMemcpy(m.d_weights_logical, m.host_weights.data(), count * 4, cudaMemcpyHostToDevice), "weights H2D");
  auto specs = weight_specs(m.arch);
  std::map<std::string, const WeightSpec *> by_name;
  for (const auto &s : specs) by_name[s.name] = &s;
  // packed buffer: same element count, each tensor 16-byte aligned
  std::vector<size_t> pk_off(specs.size());
  size_t total = 0;
  for (size_t i = 0; i < specs.size(); i++) {
    pk_off[i] = total;
    total = align_up(total + specs[i].count, 4);
  }
  cuda_check(cudaMalloc(&m.d_weights, total * 4), "cudaMalloc packed weights");
  m.device_bytes += (count + total) * 4;
  int rb = m.T == gpu::BF16 ? 1 : 0;
  std::map<std::string, float *> packed;
  for (size_t i = 0; i < specs.size(); i++) {
    const auto &s = specs[i];
    const float *src = m.d_weights_logical + s.offset;
    float *dst = m.d_weights + pk_off[i];
    bool bias = s.name.size() >= 4 && s.name.compare(s.name.size() - 4, 4, "bias") == 0;
    if (s.name.find("dw_weight") != std::string::npos)
      cuda_check(gpu::pack_dw(src, s.shape[0], s.shape[1], dst, rb, m.stream), "pack dw");
    else if (s.shape.size() == 4)
      cuda_check(gpu::pack_conv(src, s.shape[0], s.shape[1], s.shape[2], dst, rb, m.stream), "pack conv");
    else
      cuda_check(gpu::copy_round(src, (long)s.count, dst, bias ? 0 : rb, m.stream), "pack");
    packed[s.name] = dst;
  }
  m.opw.resize(m.arch.ops.size());
  for (size_t i = 0; i < m.arch.ops.size(); i++) {
    const Op &op = m.arch.ops[i];
    OpWeights &w = m.opw[i];
    auto get = [&](const std::string &suffix) -> float * {
      auto it = packed.find(op.name + "." + suffix);
      if (it == packed.end()) throw Error(ILLUMINA_BAD_WEIGHTS, "weights: " + op.name + "." + suffix + " is missing");
      return it->second;
    };
    switch (op.kind) {
      case OpKind::Conv:
      case OpKind::Pw:
      case OpKind::Lateral:
      case OpKind::Head:
        w.w = get("weight");
        w.b = get("bias");
        break;
      case OpKind::Dwpw:
        w.dw_w = get("dw_weight");
        w.dw_b = get("dw_bias");
        w.w = get("pw_weight");
        w.b = get("pw_bias");
        break;
      default: break;
    }
    if (op.kind == OpKind::Head) w.head_bias = m.host_weights[by_name[op.name + ".bias"]->offset];
  }

  // --- tensor-core weight images (from the logical weights) ---
  if (o.gemm_engine != ILLUMINA_ENGINE_TENSOR && o.gemm_engine != ILLUMINA_ENGINE_SIMT)
    throw Error(ILLUMINA_INVALID_ARG, "createDepthModel: unknown gemm engine " + std::to_string(o.gemm_engine));
  m.engine = o.gemm_engine;
  plan_head_fusion(m);
  {
    void *h = nullptr;
    cuda_check(cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped), "cudaHostAlloc error word");
    m.h_err = (volatile int *)h;
    *m.h_err = 0;
    void *d = nullptr;
    cuda_check(cudaHostGetDevicePointer(&d, h, 0), "error word device address");
    m.d_err = (int *)d;
  }
  if (o.gemm_engine == ILLUMINA_ENGINE_TENSOR) {
    cuda_check(cudaMalloc(&m.d_splitk, kSplitKBytes), "cudaMalloc split-K workspace");
    m.device_bytes += kSplitKBytes;
  }
  m.tcw.resize(m.arch.ops.size());
  m.tc_off.assign(m.arch.ops.size(), 0);
  if (m.engine == ILLUMINA_ENGINE_TENSOR) {
    size_t total_img = 0;
    std::vector<const WeightSpec *> pw_spec(m.arch.ops.size(), nullptr);
    for (size_t i = 0; i < m.arch.ops.size(); i++) {
      const Op &op = m.arch.ops[i];
      if (op.kind != OpKind::Pw && op.kind != OpKind::Dwpw && op.kind != OpKind::Lateral) continue;
      pw_spec[i] = by_name[op.name + (op.kind == OpKind::Dwpw ? ".pw_weight" : ".weight")];
      m.tcw[i] = op.kind == OpKind::Dwpw ? gpu::tc_plan_dw(m.T, pw_spec[i]->shape[0], pw_spec[i]->shape[1], op.k)
                                         : gpu::tc_plan(m.T, pw_spec[i]->shape[0], pw_spec[i]->shape[1]);
      m.tc_off[i] = total_img;
      total_img = align_up(total_img + m.tcw[i].bytes, 1024);
    }
    cuda_check(cudaMalloc(&m.d_wimg, total_img), "cudaMalloc weight images");
    cuda_check(cudaMemsetAsync(m.d_wimg, 0, total_img, m.stream), "clear weight images");
    m.device_bytes += total_img;
    for (size_t i = 0; i < m.arch.ops.size(); i++) {
      if (!pw_spec[i]) continue;
      cuda_check(gpu::tc_pack(m.T, m.d_weights_logical + pw_spec[i]->offset, m.tcw[i].N, m.tcw[i].K, m.tcw[i],
                              m.d_wimg + m.tc_off[i], m.stream),
                 "pack weight images");
      if (m.tcw[i].dw_bytes)
        cuda_check(gpu::tc_pack_dw(m.T, m.opw[i].dw_w, m.opw[i].dw_b, m.tcw[i], m.d_wimg + m.tc_off[i], m.stream),
                   "pack depthwise blocks");
    }
  }

  // --- arena: one allocation, buffers 256-byte aligned, sized for max_batch ---
  const size_t B = (size_t)m.opts.max_batch;
  m.buf_off.resize(m.plan.buffer_sizes.size());
  size_t off = 0;
  for (size_t b = 0; b < m.plan.buffer_sizes.size(); b++) {
    m.buf_off[b] = off;
    off = align_up(off + (size_t)m.plan.buffer_sizes[b] * 4 * m.elt * B, 256);
  }
  m.arena_alloc = off;
  cuda_check(cudaMalloc(&m.d_arena, off), "cudaMalloc arena");
  const int S = m.arch.input_size;
  cuda_check(cudaMalloc(&m.d_luma, sizeof(float) * B * S * S), "cudaMalloc guide");
  if (o.keep_intermediates) cuda_check(cudaMalloc(&m.d_scene, sizeof(float) * 4 * B * S * S), "cudaMalloc scene");
  for (int i = 0; i < 2; i++) {
    cuda_check(cudaMalloc(&m.d_tex[i], sizeof(float) * 4 * S * S), "cudaMalloc depth");
    cuda_check(cudaMemsetAsync(m.d_tex[i], 0, sizeof(float) * 4 * S * S, m.stream), "clear depth");
  }
  cuda_check(cudaMalloc(&m.d_stage_in, sizeof(float) * 4 * B * S * S), "cudaMalloc staging");
  cuda_check(cudaMalloc(&m.d_stage_out, sizeof(float) * B * S * S), "cudaMalloc staging");
  cuda_check(cudaMalloc(&m.d_stage_low, sizeof(float) * B * (S / 2) * (S / 2)), "cudaMalloc staging");
  m.device_bytes += off + sizeof(float) * B * S * S * (1 + 4 + 1) + sizeof(float) * B * (S / 2) * (S / 2) +
                    2 * sizeof(float) * 4 * S * S + (m.d_scene ? sizeof(float) * 4 * B * S * S : 0);
  cuda_check(cudaStreamSynchronize(m.stream), "create synchronize");
  // The logical copy is only needed for packing.
  cudaFree(m.d_weights_logical);
  m.d_weights_logical = nullptr;
  m.device_bytes -= count * 4;
  m.launches_per_forward = (int)m.arch.ops.size();
}

// Op-API helper: temporary device scratch on a stream.
struct Scratch {
  void *p = nullptr;
  cudaStream_t st;
  Scratch(size_t bytes, cudaStream_t s) : st(s) { cuda_check(cudaMallocAsync(&p, bytes, s), "cudaMallocAsync"); }
  ~Scratch() {
    if (p) cudaFreeAsync(p, st);
  }
};

void require(bool ok, const std::string &msg) {
  if (!ok) throw Error(ILLUMINA_INVALID_ARG, msg);
}

thread_local int g_op_engine = ILLUMINA_ENGINE_SIMT;

// Per-kernel entry points: run `g` (fp32, logical [N][K] weights in g.w) on
// the calling thread's engine; the tensor-core engine packs its weight images
// into temporary device memory first.
void op_gemm(const gpu::GemmOp &g, cudaStream_t st, const char *what) {
  if (g_op_engine == ILLUMINA_ENGINE_SIMT) {
    cuda_check(gpu::gemm(gpu::F32, g, st), what);
    return;
  }
  gpu::TcWeights plan = g.mode == 1 ? gpu::tc_plan_dw(gpu::F32, g.N, g.K, g.ks) : gpu::tc_plan(gpu::F32, g.N, g.K);
  Scratch img(plan.bytes, st);
  cuda_check(cudaMemsetAsync(img.p, 0, plan.bytes, st), "clear weight images");
  cuda_check(gpu::tc_pack(gpu::F32, g.w, g.N, g.K, plan, (uint8_t *)img.p, st), "pack weight images");
  if (g.mode == 1)
    cuda_check(gpu::tc_pack_dw(gpu::F32, g.dw_w, g.dw_b, plan, (uint8_t *)img.p, st), "pack depthwise blocks");
  Scratch ws(kSplitKOpBytes, st);
  gpu::GemmOp gs = g;
  gs.ws = (float *)ws.p, gs.ws_bytes = kSplitKOpBytes;
  cuda_check(gpu::tc_op(gpu::F32, gs, plan, (const uint8_t *)img.p, nullptr, st), what);
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" {

const char *illumina_last_error(void) { return g_last_error.c_str(); }
const char *illumina_version(void) { return "illumina-b200 0.1 (sm_100a)"; }

int illumina_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

illumina_status illumina_arch_json(int input_size, char *buf, size_t cap, size_t *needed) {
  ILL_TRY
  write_json(arch_to_json(build_architecture(input_size)), buf, cap, needed, 0);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_arena_json(int input_size, char *buf, size_t cap, size_t *needed) {
  ILL_TRY
  Architecture a = build_architecture(input_size);
  std::vector<std::string> ex = {"depth"};
  ArenaPlan p = plan_arena(a, ex);
  validate_arena(a, p, ex);
  write_json(arena_to_json(p), buf, cap, needed, 0);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_weights_count(int input_size, size_t *count) {
  ILL_TRY
  require(count != nullptr, "weights_count: count is null");
  *count = weight_count(build_architecture(input_size));
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_weights_synthesize(int input_size, uint32_t seed, float *out, size_t count) {
  ILL_TRY
  Architecture a = build_architecture(input_size);
  require(out && count == weight_count(a), "synthesizeWeights: output must hold " + std::to_string(weight_count(a)) + " floats");
  auto blob = synthesize_weights(a, seed);
  std::memcpy(out, blob.data(), blob.size() * 4);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_weights_parse(int input_size, const void *bytes, size_t len, float *out, size_t count) {
  ILL_TRY
  Architecture a = build_architecture(input_size);
  require(out && count == weight_count(a), "parseWeights: output must hold " + std::to_string(weight_count(a)) + " floats");
  require(bytes != nullptr || len == 0, "parseWeights: bytes is null");
  auto blob = parse_weights(a, (const uint8_t *)bytes, len);
  std::memcpy(out, blob.data(), blob.size() * 4);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_weights_serialize(int input_size, const float *blob, size_t count, void *out, size_t cap,
                                           size_t *needed) {
  ILL_TRY
  Architecture a = build_architecture(input_size);
  require(blob != nullptr, "serializeWeights: blob is null");
  auto bytes = serialize_weights(a, blob, count);
  if (needed) *needed = bytes.size();
  if (out) {
    require(cap >= bytes.size(), "serializeWeights: output buffer too small");
    std::memcpy(out, bytes.data(), bytes.size());
  }
  return ILLUMINA_OK;
  ILL_CATCH
}

double illumina_half_to_float(uint16_t h) { return half_to_float(h); }

void illumina_model_options_default(illumina_model_options *o) {
  if (!o) return;
  std::memset(o, 0, sizeof *o);
  o->input_size = 448;
  o->device = 0;
  o->max_batch = 1;
  o->precision = ILLUMINA_PRECISION_F32;
  o->decode_srgb = 1;
  o->exposure = 1.0f;
  o->range_sigma = 0.12f;
  o->temporal_base = 0.35f;
  o->temporal_sensitivity = 3.0f;
  o->synth_seed = 1;
  o->gemm_engine = ILLUMINA_ENGINE_TENSOR;
}

illumina_status illumina_model_create(const illumina_model_options *opts, illumina_model **out) {
  ILL_TRY
  require(opts && out, "createDepthModel: null argument");
  *out = nullptr;
  auto m = std::make_unique<illumina_model>();
  m->device = -1;
  build_model(*m, *opts);
  *out = m.release();
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_destroy(illumina_model *model) {
  delete model;
  return ILLUMINA_OK;
}

illumina_status illumina_model_set_exposure(illumina_model *m, float exposure) {
  ILL_TRY
  require(m, "setExposure: null model");
  if (m->exposure != exposure) m->clear_graphs();
  m->exposure = exposure;
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_set_temporal(illumina_model *m, float base, float sens, float sigma) {
  ILL_TRY
  require(m, "setTemporal: null model");
  if (m->base_alpha != base || m->sensitivity != sens || m->range_sigma != sigma) m->clear_graphs();
  m->base_alpha = base, m->sensitivity = sens, m->range_sigma = sigma;
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_forward(illumina_model *m, const float *frames, int n, int layout, float *disparity,
                                 float *depth_low, void *stream) {
  ILL_TRY
  require(m, "forward: null model");
  run_forward(*m, frames, n, layout, disparity, depth_low, (cudaStream_t)stream, 0);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_forward_async(illumina_model *m, const float *frames, int n, int layout, float *disparity,
                                       void *stream) {
  ILL_TRY
  require(m, "forwardAsync: null model");
  run_forward_async(*m, frames, n, layout, disparity, (cudaStream_t)stream);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_forward_source_async(illumina_model *m, const uint8_t *rgba8, int n, int src_w, int src_h,
                                              const float *uv_scale, const float *uv_offset, int mirror,
                                              float *disparity, void *stream) {
  ILL_TRY
  require(m, "forwardSourceAsync: null model");
  const AsyncSource src{rgba8, src_w, src_h, mirror, uv_scale, uv_offset};
  run_forward_async(*m, nullptr, n, ILLUMINA_FRAME_RGB_PLANAR, disparity, (cudaStream_t)stream, &src);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_forward_source(illumina_model *m, const uint8_t *rgba8, int n, int src_w, int src_h,
                                        const float *uv_scale, const float *uv_offset, int mirror, float *disparity,
                                        void *stream) {
  ILL_TRY
  require(m, "forwardSource: null model");
  run_forward_source(*m, rgba8, n, src_w, src_h, uv_scale, uv_offset, mirror, disparity, (cudaStream_t)stream);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_forward_input(illumina_model *m, const float *input, int n, float *disparity,
                                       float *depth_low) {
  ILL_TRY
  require(m && input, "forwardInput: null argument");
  require(m->T == gpu::F32, "forwardInput: the network input is given in fp32; use an fp32 model");
  require(n >= 1 && n <= m->opts.max_batch, "forwardInput: batch " + std::to_string(n) + " outside [1, " +
                                                std::to_string(m->opts.max_batch) + "]");
  cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
  check_timeout(*m, "in an earlier call on this model");
  const int S = m->arch.input_size;
  const size_t px = (size_t)n * S * S;
  float *in = (float *)m->tensor("input");
  cuda_check(cudaMemcpyAsync(in, input, sizeof(float) * 4 * px, cudaMemcpyDefault, m->stream), "input copy");
  // the bilateral guide is the input's unnormalised luminance (channel 3)
  cuda_check(gpu::input_luma(in, (long)px, m->d_luma, m->stream), "guide");
  enqueue_forward(*m, n, nullptr, ILLUMINA_FRAME_RGB_PLANAR, m->d_stage_out, m->d_stage_low, nullptr, nullptr,
                  nullptr, nullptr, true);
  if (disparity)
    cuda_check(cudaMemcpyAsync(disparity, m->d_stage_out, sizeof(float) * px, cudaMemcpyDefault, m->stream),
               "disparity copy");
  if (depth_low)
    cuda_check(cudaMemcpyAsync(depth_low, m->d_stage_low, sizeof(float) * px / 4, cudaMemcpyDefault, m->stream),
               "depth_low copy");
  cuda_check(cudaStreamSynchronize(m->stream), "synchronize");
  check_timeout(*m, "in this call");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_record(illumina_model *m, const float *frame, int layout, void *stream) {
  ILL_TRY
  require(m, "record: null model");
  run_forward(*m, frame, 1, layout, nullptr, nullptr, (cudaStream_t)stream, 1);
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_sync(illumina_model *m) {
  ILL_TRY
  require(m, "sync: null model");
  cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
  cuda_check(cudaStreamSynchronize(m->stream), "synchronize");
  cuda_check(cudaStreamSynchronize(m->copy_in), "synchronize");
  cuda_check(cudaStreamSynchronize(m->copy_out), "synchronize");
  check_timeout(*m, "in a forward queued since the last check");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_set_wait_limit(illumina_model *m, long long cycles) {
  ILL_TRY
  require(m && cycles >= 0, "setWaitLimit: bad arguments");
  cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
  cuda_check(cudaStreamSynchronize(m->stream), "synchronize");
  m->wait_cycles = cycles;
  m->clear_graphs();  // the limit is a kernel parameter of the captured launches
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_swap_history(illumina_model *m) {
  ILL_TRY
  require(m, "swapHistory: null model");
  m->history_index = 1 - m->history_index;
  return ILLUMINA_OK;
  ILL_CATCH
}

int illumina_model_output_parity(const illumina_model *m) { return m ? 1 - m->history_index : -1; }
int illumina_model_fresh_parity(const illumina_model *m) { return m ? m->last_written : -1; }

illumina_status illumina_model_depth_slot(illumina_model *m, int index, const float **ptr) {
  ILL_TRY
  require(m && ptr, "debugDepth: null argument");
  *ptr = m->d_tex[index == 0 ? 0 : 1];
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_debug_tensor_frame(illumina_model *m, const char *name, int frame, float *out,
                                                  size_t cap, int *h, int *w, int *c, int *live_at_end) {
  ILL_TRY
  require(m && name, "debugTensor: null argument");
  std::string n(name);
  require(frame >= 0 && frame < m->opts.max_batch,
          "debugTensor: frame " + std::to_string(frame) + " outside [0, " + std::to_string(m->opts.max_batch) + ")");
  if (n == "scene_color") {
    // the preprocess's second output (linear exposed colour, alpha 1), kept
    // only by a keep-intermediates model
    const int S = m->arch.input_size;
    require(m->d_scene != nullptr, "debugTensor: scene_color is kept only by a keepIntermediates model");
    if (h) *h = S;
    if (w) *w = S;
    if (c) *c = 4;
    if (live_at_end) *live_at_end = 1;
    if (!out) return ILLUMINA_OK;
    const size_t count = (size_t)4 * S * S;
    require(cap >= count, "debugTensor: output holds " + std::to_string(cap) + " floats, tensor needs " +
                              std::to_string(count));
    cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
    cuda_check(cudaMemcpyAsync(out, m->d_scene + (size_t)frame * count, sizeof(float) * count, cudaMemcpyDefault,
                               m->stream),
               "debugTensor copy");
    cuda_check(cudaStreamSynchronize(m->stream), "debugTensor copy");
    return ILLUMINA_OK;
  }
  auto ts = m->arch.tensors.find(n);
  auto as = m->plan.assignment.find(n);
  if (ts == m->arch.tensors.end() || as == m->plan.assignment.end())
    throw Error(ILLUMINA_INVALID_ARG, "debugTensor: unknown tensor " + n);
  const TensorShape &s = ts->second;
  if (h) *h = s.h;
  if (w) *w = s.w;
  if (c) *c = s.c;
  if (live_at_end) *live_at_end = tensor_live_at_end(*m, n) ? 1 : 0;
  if (!out) return ILLUMINA_OK;
  cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
  long count = s.elems();
  require(cap >= (size_t)count, "debugTensor: output holds " + std::to_string(cap) + " floats, tensor needs " +
                                    std::to_string(count));
  float *tmp = nullptr;
  cuda_check(cudaMalloc(&tmp, sizeof(float) * count), "cudaMalloc");
  cudaError_t e;
  // frames are stored one after another: depth_low as one fp32 channel per
  // pixel, every other tensor as h x w x c elements of the model's type
  const char *base = (const char *)m->tensor(n);
  if (n == "depth_low")
    e = gpu::expand4((const float *)(base + (size_t)frame * s.h * s.w * sizeof(float)), (long)s.h * s.w, tmp,
                     m->stream);
  else
    e = gpu::to_f32(m->T, base + (size_t)frame * count * m->elt, count, tmp, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, tmp, sizeof(float) * count, cudaMemcpyDefault, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  cudaFree(tmp);
  cuda_check(e, "debugTensor copy");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_debug_tensor(illumina_model *m, const char *name, float *out, size_t cap, int *h,
                                            int *w, int *c, int *live_at_end) {
  return illumina_model_debug_tensor_frame(m, name, 0, out, cap, h, w, c, live_at_end);
}

illumina_status illumina_model_stats(const illumina_model *m, illumina_stats *out) {
  ILL_TRY
  require(m && out, "stats: null argument");
  out->dispatches = (int)m->arch.ops.size();
  out->launches = m->launches_per_forward;
  out->arena_bytes = (size_t)m->plan.total_bytes;
  out->naive_arena_bytes = (size_t)m->plan.naive_bytes;
  out->weight_bytes = m->host_weights.size() * 4;
  out->device_bytes = m->device_bytes;
  out->max_batch = m->opts.max_batch;
  out->precision = m->opts.precision;
  out->input_size = m->arch.input_size;
  out->gemm_engine = m->engine;
  cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
  cuda_check(cudaStreamSynchronize(m->stream), "synchronize");
  out->device_error = m->h_err ? *m->h_err : 0;
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_model_profile(illumina_model *m, const float *frames, int n, int layout, int reps,
                                       float *op_ms, int cap) {
  ILL_TRY
  require(m && frames && op_ms, "profile: null argument");
  require(n >= 1 && n <= m->opts.max_batch, "profile: batch outside [1, max_batch]");
  require(reps >= 1, "profile: reps must be positive");
  require(is_device_ptr(frames), "profile: frames must be device memory");
  const size_t nops = m->arch.ops.size();
  require(cap >= (int)nops, "profile: op_ms must hold " + std::to_string(nops) + " floats");
  cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
  std::vector<cudaEvent_t> ev(nops + 1);
  for (auto &e : ev) cuda_check(cudaEventCreate(&e), "event create");
  std::vector<double> acc(nops, 0.0);
  cudaError_t err = cudaSuccess;
  try {
    for (int r = 0; r < reps; r++) {
      enqueue_forward(*m, n, frames, layout, m->d_stage_out, nullptr, nullptr, nullptr, &ev);
      cuda_check(cudaEventSynchronize(ev[nops]), "profile sync");
      for (size_t i = 0; i < nops; i++) {
        float ms = 0;
        cuda_check(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "elapsed");
        acc[i] += ms;
      }
    }
  } catch (...) {
    for (auto &e : ev) cudaEventDestroy(e);
    throw;
  }
  for (auto &e : ev) cudaEventDestroy(e);
  cuda_check(err, "profile");
  for (size_t i = 0; i < nops; i++) op_ms[i] = (float)(acc[i] / reps);
  return ILLUMINA_OK;
  ILL_CATCH
}

// ---- per-kernel entry points -------------------------------------------------

illumina_status illumina_set_op_engine(int engine) {
  ILL_TRY
  require(engine == ILLUMINA_ENGINE_TENSOR || engine == ILLUMINA_ENGINE_SIMT, "set_op_engine: unknown engine");
  g_op_engine = engine;
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_pointwise(const float *src, long pixels, int in_c, const float *w, const float *b,
                                      int out_c, int act, const float *res, float *dst, void *stream) {
  ILL_TRY
  require(src && w && b && dst, "pointwise: null pointer");
  require(in_c > 0 && out_c > 0 && in_c % 4 == 0 && out_c % 4 == 0, "pointwise: channels must be multiples of 4");
  require(act >= 0 && act <= 3, "pointwise: unknown activation");
  gpu::GemmOp g;
  g.mode = 0, g.src = src, g.w = w, g.bias = b, g.res = res, g.dst = dst, g.M = pixels, g.N = out_c, g.K = in_c;
  g.act = act;
  op_gemm(g, (cudaStream_t)stream, "pointwise");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_dwpw(const float *src, int in_h, int in_w, int in_c, const float *dw_w, const float *dw_b,
                                 int mid_act, const float *pw_w, const float *pw_b, int out_c, int k, int stride,
                                 int act, const float *res, float *dst, void *stream) {
  ILL_TRY
  require(src && dw_w && dw_b && pw_w && pw_b && dst, "dwpw: null pointer");
  require(in_c % 4 == 0 && out_c % 4 == 0 && in_c > 0 && out_c > 0, "dwpw: channels must be multiples of 4");
  require(k == 3 || k == 5, "dwpw: kernel size must be 3 or 5");
  require(stride == 1 || stride == 2, "dwpw: stride must be 1 or 2");
  require(act >= 0 && act <= 3 && mid_act >= 0 && mid_act <= 3, "dwpw: unknown activation");
  cudaStream_t st = (cudaStream_t)stream;
  int pad = (k - 1) >> 1;
  int oh = (in_h + 2 * pad - k) / stride + 1, ow = (in_w + 2 * pad - k) / stride + 1;
  Scratch pk(sizeof(float) * in_c * k * k, st);
  cuda_check(gpu::pack_dw(dw_w, in_c, k, (float *)pk.p, 0, st), "pack dw");
  gpu::GemmOp g;
  g.mode = 1, g.src = src, g.w = pw_w, g.bias = pw_b, g.res = res, g.dst = dst;
  g.H = in_h, g.W = in_w, g.OH = oh, g.OW = ow, g.M = (long)oh * ow, g.N = out_c, g.K = in_c;
  g.act = act, g.mid_act = mid_act, g.ks = k, g.stride = stride, g.dw_w = (const float *)pk.p, g.dw_b = dw_b;
  op_gemm(g, st, "dwpw");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_conv(const float *src, int in_h, int in_w, int in_c, const float *w, const float *b,
                                 int out_c, int k, int stride, int act, float *dst, void *stream) {
  ILL_TRY
  require(src && w && b && dst, "conv: null pointer");
  require(in_c % 4 == 0 && out_c % 4 == 0 && in_c > 0 && out_c > 0, "conv: channels must be multiples of 4");
  require(k >= 1 && k % 2 == 1 && stride >= 1, "conv: odd kernel size and positive stride required");
  require(act >= 0 && act <= 3, "conv: unknown activation");
  cudaStream_t st = (cudaStream_t)stream;
  Scratch pk(sizeof(float) * out_c * in_c * k * k, st);
  cuda_check(gpu::pack_conv(w, out_c, in_c, k, (float *)pk.p, 0, st), "pack conv");
  cuda_check(gpu::conv(gpu::F32, src, 1, in_h, in_w, in_c, (const float *)pk.p, b, out_c, k, stride, act, dst, st),
             "conv");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_lateral(const float *coarse, int ch, int cw, const float *skip, int skip_c, const float *w,
                                    const float *b, int out_c, int act, float *dst, void *stream) {
  ILL_TRY
  require(coarse && skip && w && b && dst, "lateral: null pointer");
  require(skip_c % 4 == 0 && out_c % 4 == 0 && skip_c > 0 && out_c > 0, "lateral: channels must be multiples of 4");
  require(act >= 0 && act <= 3, "lateral: unknown activation");
  gpu::GemmOp g;
  g.mode = 2, g.src = skip, g.coarse = coarse, g.w = w, g.bias = b, g.dst = dst;
  g.OH = 2 * ch, g.OW = 2 * cw, g.M = 4L * ch * cw, g.N = out_c, g.K = skip_c, g.act = act;
  op_gemm(g, (cudaStream_t)stream, "lateral");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_head(const float *src, long pixels, int in_c, const float *w, float b, float *dst4,
                                 void *stream) {
  ILL_TRY
  require(src && w && dst4, "head: null pointer");
  require(in_c % 4 == 0 && in_c > 0, "head: channels must be a multiple of 4");
  cuda_check(gpu::head(gpu::F32, src, pixels, in_c, w, b, nullptr, dst4, (cudaStream_t)stream), "head");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_preprocess(const float *frames, int n, int layout, int size, int decode_srgb,
                                       float exposure, float *input, float *scene_color, void *stream) {
  ILL_TRY
  require(frames && input, "preprocess: null pointer");
  require(layout == 0 || layout == 1, "preprocess: unknown layout");
  gpu::PreprocessParams p;
  const double mean[3] = {0.485, 0.456, 0.406}, stdv[3] = {0.229, 0.224, 0.225};
  for (int i = 0; i < 3; i++) p.mean[i] = (float)mean[i], p.std[i] = (float)stdv[i], p.inv_std[i] = (float)(1 / stdv[i]);
  p.exposure = exposure;
  p.decode_srgb = decode_srgb ? 1 : 0;
  cuda_check(gpu::preprocess(gpu::F32, frames, layout, n, size, p, input, nullptr, scene_color, (cudaStream_t)stream),
             "preprocess");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_op_bilateral(const float *low, int lh, int lw, int low_c, const float *guide, int guide_c,
                                      float range_sigma, float *dst, void *stream) {
  ILL_TRY
  require(low && guide && dst, "bilateral: null pointer");
  require(lh > 0 && lw > 0 && low_c >= 1 && guide_c >= 3, "bilateral: bad shape");
  cuda_check(gpu::bilateral_strided(low, lh, lw, low_c, guide, guide_c, range_sigma, dst, (cudaStream_t)stream),
             "bilateral");
  return ILLUMINA_OK;
  ILL_CATCH
}

// ---- lighting ------------------------------------------------------------------

void illumina_shading_settings_default(illumina_shading_settings *s) {
  if (!s) return;
  std::memset(s, 0, sizeof *s);
  s->fov_y = (float)(58.0 * M_PI / 180.0);
  s->near_m = 0.35f, s->far_m = 14.0f;
  s->ao_strength = 0.85f, s->shadow_strength = 0.8f, s->volumetric = 0.35f, s->exposure = 1.15f;
  s->ambient[0] = 0.16f, s->ambient[1] = 0.2f, s->ambient[2] = 0.3f;
  s->ambient_intensity = 0.5f, s->roughness = 0.55f, s->fog_density = 0.028f;
  s->fog_color[0] = 0.05f, s->fog_color[1] = 0.07f, s->fog_color[2] = 0.12f;
  s->specular = 0.6f, s->normal_strength = 1.0f, s->albedo_mix = 1.0f, s->contact_shadow_length = 0.8f;
  s->ao_radius_pixels = 14.0f;
  s->tone_map = 0;
  s->contrast = 1.04f, s->saturation = 1.06f, s->vignette = 0.35f;
  s->debug_view = 0;
}

illumina_status illumina_shade(const float *disparity, int dw, int dh, int dch, const float *albedo, int aw, int ah,
                               const illumina_light *lights, const illumina_shading_settings *s, uint32_t frame,
                               const illumina_shade_steps *steps, int out_w, int out_h, float *hdr, uint8_t *rgba8,
                               void *stream) {
  ILL_TRY
  require(disparity && albedo && lights && s, "shade: null pointer");
  require(dw > 0 && dh > 0 && aw > 0 && ah > 0 && out_w > 0 && out_h > 0, "shade: sizes must be positive");
  require(dch == 1 || dch == 4, "shade: disparity_channels must be 1 or 4");
  require(s->debug_view >= 0 && s->debug_view <= 4, "shade: unknown debug view");
  // Renderer.update (renderer.ts:206-231)
  gpu::ShadeParams P;
  float cam[4] = {std::tan(s->fov_y / 2), (float)out_w / (float)out_h, s->near_m, s->far_m};
  float tog[4] = {s->ao_strength, s->shadow_strength, s->volumetric, s->exposure};
  float amb[4] = {s->ambient[0], s->ambient[1], s->ambient[2], s->ambient_intensity};
  float misc[4] = {(float)(frame % 4096), s->roughness, s->fog_density, s->normal_strength};
  float fog[4] = {s->fog_color[0], s->fog_color[1], s->fog_color[2], s->specular};
  float size[4] = {(float)out_w, (float)out_h, (float)dw, (float)dh};
  float dbg[4] = {(float)s->debug_view, s->albedo_mix, s->contact_shadow_length, s->ao_radius_pixels};
  float grade[4] = {(float)(s->tone_map == 0 ? 0 : 1), s->contrast, s->saturation, s->vignette};
  std::memcpy(P.camera, cam, 16), std::memcpy(P.toggles, tog, 16), std::memcpy(P.ambient, amb, 16);
  std::memcpy(P.misc, misc, 16), std::memcpy(P.fog, fog, 16), std::memcpy(P.size, size, 16);
  std::memcpy(P.debug, dbg, 16), std::memcpy(P.grade, grade, 16);
  gpu::ShadeSteps st{12, 6, 4, 10};
  if (steps) {
    require(steps->contact > 0 && steps->ao_dirs > 0 && steps->ao_steps > 0 && steps->volumetric > 0,
            "shade: step counts must be positive");
    st = gpu::ShadeSteps{steps->contact, steps->ao_dirs, steps->ao_steps, steps->volumetric};
  }
  gpu::ShadeLight L[8];
  std::memcpy(L, lights, sizeof(L));
  cuda_check(gpu::shade(disparity, dw, dh, dch, albedo, aw, ah, L, P, st, out_w, out_h, hdr, rgba8, (cudaStream_t)stream),
             "shade");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_resize_bilinear(const float *src, int sw, int sh, float *dst, int dw, int dh, void *stream) {
  ILL_TRY
  require(src && dst && sw > 0 && sh > 0 && dw > 0 && dh > 0, "resize: bad arguments");
  cuda_check(gpu::resize_bilinear(src, sw, sh, dst, dw, dh, (cudaStream_t)stream), "resize");
  return ILLUMINA_OK;
  ILL_CATCH
}

// ---- 8-bit source sampling ---------------------------------------------------------

illumina_status illumina_sample_source(const uint8_t *rgba8, int n, int src_w, int src_h, const float *uv_scale,
                                       const float *uv_offset, int mirror, int size, float *frames, void *stream) {
  ILL_TRY
  require(n >= 0 && n <= 65535, "sample_source: n must be in [0, 65535]");
  require(src_w > 0 && src_h > 0 && size > 0, "sample_source: bad size");
  require(n == 0 || (rgba8 && frames), "sample_source: null pointer");
  require((reinterpret_cast<uintptr_t>(rgba8) & 3) == 0, "sample_source: rgba8 must be 4-byte aligned");
  const float one[2] = {1.0f, 1.0f}, zero[2] = {0.0f, 0.0f};
  cuda_check(gpu::sample_source(rgba8, n, src_w, src_h, uv_scale ? uv_scale : one, uv_offset ? uv_offset : zero,
                                mirror ? 1 : 0, size, frames, (cudaStream_t)stream),
             "sample_source");
  return ILLUMINA_OK;
  ILL_CATCH
}

void illumina_crop_transform(int width, int height, float out[4]) {
  if (!out) return;
  if (width <= 0 || height <= 0) {
    out[0] = 1.0f, out[1] = 1.0f, out[2] = 0.0f, out[3] = 0.0f;
    return;
  }
  const double sx = width > height ? (double)height / width : 1.0;
  const double sy = height > width ? (double)width / height : 1.0;
  out[0] = (float)sx, out[1] = (float)sy, out[2] = (float)((1 - sx) / 2), out[3] = (float)((1 - sy) / 2);
}

// ---- procedural scene and depth metrics ------------------------------------------

static_assert(sizeof(illumina_scene_params) == sizeof(gpu::SceneParams), "scene params layout");
static_assert(sizeof(illumina_depth_metrics) == sizeof(gpu::DepthMetrics), "depth metrics layout");

void illumina_scene_params_initial(illumina_scene_params *p) {
  if (!p) return;
  const float tan_half = (float)std::tan((58.0 * M_PI) / 180.0 / 2.0);
  const float v[12] = {0.0f, 0.35f, 0.6f, 0.0f, 0.0f, -0.15f, -3.0f, tan_half, 1.0f, 30.0f, 0.9f, 0.0f};
  std::memcpy(p, v, sizeof(v));
}

void illumina_scene_params_update(illumina_scene_params *p, double time, int orbit) {
  if (!p) return;
  const double angle = orbit ? std::sin(time * 0.18) * 0.5 : 0.0;
  const double height = 0.35 + (orbit ? std::sin(time * 0.11) * 0.12 : 0.0);
  const float v[12] = {(float)(std::sin(angle) * 1.4), (float)height, (float)(0.6 + std::cos(angle) * 0.3),
                       (float)time, 0.0f, -0.15f, -3.0f, (float)std::tan((58.0 * M_PI) / 180.0 / 2.0),
                       1.0f, 30.0f, (float)(0.9 + time * 0.03), 0.0f};
  std::memcpy(p, v, sizeof(v));
}

illumina_status illumina_scene_render(const illumina_scene_params *params, int n, int width, int height, float *rgb,
                                      uint8_t *rgba8, float *truth, void *stream) {
  ILL_TRY
  require(n >= 0 && width > 0 && height > 0, "scene_render: bad size");
  require(n == 0 || params, "scene_render: params is null");
  cuda_check(gpu::scene_render(reinterpret_cast<const gpu::SceneParams *>(params), n, width, height, rgb, rgba8,
                               truth, (cudaStream_t)stream),
             "scene_render");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_evaluate_depth(const float *pred, int pred_channels, const float *truth, int n, int width,
                                        int height, illumina_depth_metrics *out, void *stream) {
  ILL_TRY
  require(n >= 0 && width > 0 && height > 0, "evaluate_depth: bad size");
  require(pred_channels >= 1, "evaluate_depth: pred_channels must be >= 1");
  require(n == 0 || (pred && truth && out), "evaluate_depth: null pointer");
  cuda_check(gpu::evaluate_depth(pred, pred_channels, truth, n, (long)width * height,
                                 reinterpret_cast<gpu::DepthMetrics *>(out), (cudaStream_t)stream),
             "evaluate_depth");
  return ILLUMINA_OK;
  ILL_CATCH
}

// ---- workloads -------------------------------------------------------------------

illumina_status illumina_generate_frames(int kind, uint32_t seed0, int n, int size, float *out, void *stream) {
  ILL_TRY
  require(out && n >= 0 && size > 0, "generate_frames: bad arguments");
  require(kind == ILLUMINA_FRAMES_UNIFORM || kind == ILLUMINA_FRAMES_BLOBS, "generate_frames: unknown kind");
  cuda_check(gpu::generate_frames(kind, seed0, n, size, out, (cudaStream_t)stream), "generate_frames");
  return ILLUMINA_OK;
  ILL_CATCH
}

illumina_status illumina_checksums(const float *maps, int n, long count, uint64_t *sum64, double *fsum, void *stream) {
  ILL_TRY
  require(maps && sum64 && fsum && n >= 0 && count > 0, "checksums: bad arguments");
  cuda_check(gpu::checksums(maps, n, count, sum64, fsum, (cudaStream_t)stream), "checksums");
  return ILLUMINA_OK;
  ILL_CATCH
}

}  // extern "C"
