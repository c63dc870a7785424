// C-ABI runtime of libemx_b200.so: plan parsing, device arena, weight upload,
// host/device I/O staging and in-order kernel dispatch.  See include/emx_b200.h.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "emx_b200.h"
#include "host_util.h"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CUDA_TRY(call, what)                                                                  \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) return set_error(EMX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e_)); \
  } while (0)

struct KernelEntry {
  uint32_t id;
  emx::PrepareFn prepare;
  emx::LaunchFn launch;
  const char* name;
};

const KernelEntry kKernels[] = {
    {emx::K_PAD_NHWC, nullptr, emx::launch_pad_nhwc, "pad_nhwc"},
    {emx::K_QCONV_TC, emx::prepare_qconv_tc, emx::launch_qconv_tc, "qconv_tc"},
    {emx::K_QCONV_GENERIC, nullptr, emx::launch_qconv_generic, "qconv_generic"},
    {emx::K_QLINEAR_ADD, nullptr, emx::launch_qlinear_add, "qlinear_add"},
    {emx::K_GEMM_F32, emx::prepare_gemm_f32, emx::launch_gemm_f32, "gemm_f32"},
    {emx::K_RELU_F32, nullptr, emx::launch_relu_f32, "relu_f32"},
    {emx::K_NBITS_GEMM, emx::prepare_nbits, emx::launch_nbits, "nbits_gemm"},
    {emx::K_NBITS_I8, emx::prepare_nbits_i8, emx::launch_nbits_i8, "nbits_i8"},
    {emx::K_SWISH_F16, emx::prepare_swish_f16, emx::launch_swish_f16, "swish_f16"},
    {emx::K_MUL_F16, nullptr, emx::launch_mul_f16, "mul_f16"},
    {emx::K_LSTM_F32, emx::prepare_lstm_f32, emx::launch_lstm_f32, "lstm_f32"},
    {emx::K_ATTENTION_F16, emx::prepare_attention, emx::launch_attention, "attention_f16"},
    {emx::K_ATTENTION_TC, emx::prepare_attention_tc, emx::launch_attention_tc, "attention_tc"},
    {emx::K_COPY, nullptr, emx::launch_copy, "copy"},
    {emx::K_TRANSPOSE, nullptr, emx::launch_transpose, "transpose"},
    {emx::K_MAXPOOL, nullptr, emx::launch_maxpool, "maxpool"},
    {emx::K_QLINEAR_AVGPOOL, nullptr, emx::launch_qlinear_avgpool, "qlinear_avgpool"},
    {emx::K_QLINEAR_SOFTMAX, nullptr, emx::launch_qlinear_softmax, "qlinear_softmax"},
    {emx::K_QLINEAR_MATMUL, emx::prepare_qmatmul, emx::launch_qmatmul, "qlinear_matmul"},
    {emx::K_MATMUL_INTEGER, emx::prepare_qmatmul, emx::launch_qmatmul, "matmul_integer"},
    {emx::K_CONV_F32, nullptr, emx::launch_conv_f32, "conv_f32"},
    {emx::K_SOFTMAX_F32, nullptr, emx::launch_softmax_f32, "softmax_f32"},
    {emx::K_QUANTIZE_LINEAR, nullptr, emx::launch_quant, "quantize_linear"},
    {emx::K_DEQUANTIZE_LINEAR, nullptr, emx::launch_quant, "dequantize_linear"},
};

const KernelEntry* find_kernel(uint32_t id) {
  for (const auto& k : kKernels)
    if (k.id == id) return &k;
  return nullptr;
}

}  // namespace

// Lets other translation units of the library report through emx_b200_last_error.
int emx_report_error(int code, const char* msg) { return set_error(code, "%s", msg); }

struct emx_plan {
  int device = 0;
  int num_sms = 0;
  PlanHeader hdr{};
  std::vector<PlanTensor> tensors;
  std::vector<uint32_t> inputs, outputs;
  std::vector<PlanOp> ops;
  std::vector<emx::OpState> states;
  std::vector<const KernelEntry*> entries;
  void* d_weights = nullptr;
  void* d_arena = nullptr;
  int* d_error = nullptr;
  cudaStream_t own_stream = nullptr;
  cudaStream_t last_stream = nullptr;
  std::vector<void*> ptrs;  // per-tensor device pointer (I/O re-resolved each run)
  int64_t launches_total = 0;
  int64_t launches_last = -1;
  // host outputs pending a device->host copy: (host dst, staging src, bytes)
  struct Pending { void* host; const void* dev; size_t bytes; };
  std::vector<Pending> pending;
  // per-op timing
  bool profiling = false;
  bool events_pending = false;
  std::vector<cudaEvent_t> ev_begin, ev_end;
  std::vector<double> op_ms;
  int64_t profiled_runs = 0;
  // CUDA graphs of the op sequence, keyed by the resolved I/O pointers
  struct GraphEntry {
    std::vector<void*> key;
    int64_t batch = 0;
    bool profiling = false;
    int launches = 0;
    uint64_t last_use = 0;
    cudaGraphExec_t exec = nullptr;
  };
  bool use_graphs = true;
  std::vector<GraphEntry> graphs;
  int fault = 0;  // failure-detection test hooks (emx_b200_set_fault)
  uint64_t graph_clock = 0;
  // host-mapped release flag for the profiling hold kernel
  int* h_hold = nullptr;
  int* d_hold = nullptr;
  int hold_seq = 0;
  // pipelined host I/O: the batch is split into io_chunks slices whose
  // upload, kernels and download run on three streams joined by events
  int io_chunks = 4;
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  std::vector<cudaEvent_t> ev_in, ev_comp;
  cudaEvent_t ev_start = nullptr, ev_done = nullptr;
  void* d_io = nullptr;           // dedicated full-batch staging of every I/O tensor (never aliased)
  std::vector<size_t> io_off;     // per I/O tensor (inputs, then outputs): offset into d_io
  std::vector<int> in_kind, out_kind;  // this run's buffers: MEM_DEVICE / MEM_PINNED / MEM_PAGEABLE
  // overlapped runs (opt-in): runs with page-locked host buffers alternate two
  // staging sets, so run k+1's upload and run k-1's download overlap run k's
  // kernels; the caller's stream does not wait for the downloads
  bool io_overlap = false;
  void* d_io2[2] = {nullptr, nullptr};
  cudaEvent_t ov_h2d[2] = {nullptr, nullptr}, ov_comp[2] = {nullptr, nullptr}, ov_d2h[2] = {nullptr, nullptr};
  uint64_t ov_seq = 0;
  cudaEvent_t ov_last = nullptr;  // download-complete event of the latest overlapped run
};

namespace {

size_t dtype_size(uint32_t dt) {
  switch (dt) {
    case EMX_U8: case EMX_I8: return 1;
    case EMX_F16: return 2;
    case EMX_F32: case EMX_I32: return 4;
    case EMX_I64: case EMX_F64: return 8;
    default: return 0;
  }
}

int parse_plan(emx_plan* p, const void* blob, size_t len) {
  const uint8_t* b = static_cast<const uint8_t*>(blob);
  if (!blob || len < sizeof(PlanHeader)) return set_error(EMX_ERR_PLAN_FORMAT, "plan blob too short (%zu bytes)", len);
  memcpy(&p->hdr, b, sizeof(PlanHeader));
  const PlanHeader& h = p->hdr;
  if (h.magic != EMX_PLAN_MAGIC) return set_error(EMX_ERR_PLAN_FORMAT, "bad plan magic 0x%08x", h.magic);
  if (h.version != EMX_PLAN_VERSION)
    return set_error(EMX_ERR_PLAN_FORMAT, "plan version %u, library expects %u", h.version, EMX_PLAN_VERSION);
  if (h.n_tensors > (1u << 20) || h.n_ops > (1u << 20) || h.n_inputs > h.n_tensors || h.n_outputs > h.n_tensors)
    return set_error(EMX_ERR_PLAN_FORMAT, "implausible plan counts");
  const size_t in_slots = (h.n_inputs + 1) & ~1u, out_slots = (h.n_outputs + 1) & ~1u;
  const size_t need = sizeof(PlanHeader) + (size_t)h.n_tensors * sizeof(PlanTensor) + (in_slots + out_slots) * 4 +
                      (size_t)h.n_ops * sizeof(PlanOp);
  if (len != need) return set_error(EMX_ERR_PLAN_FORMAT, "plan blob is %zu bytes, header implies %zu", len, need);
  size_t off = sizeof(PlanHeader);
  p->tensors.resize(h.n_tensors);
  memcpy(p->tensors.data(), b + off, h.n_tensors * sizeof(PlanTensor));
  off += h.n_tensors * sizeof(PlanTensor);
  p->inputs.resize(h.n_inputs);
  memcpy(p->inputs.data(), b + off, h.n_inputs * 4);
  off += in_slots * 4;
  p->outputs.resize(h.n_outputs);
  memcpy(p->outputs.data(), b + off, h.n_outputs * 4);
  off += out_slots * 4;
  p->ops.resize(h.n_ops);
  memcpy(p->ops.data(), b + off, h.n_ops * sizeof(PlanOp));
  // validate every reference
  for (size_t i = 0; i < p->tensors.size(); ++i) {
    const PlanTensor& t = p->tensors[i];
    const uint64_t limit = t.kind == EMX_T_WEIGHT ? h.weight_bytes : h.arena_bytes;
    if (t.kind > EMX_T_TEMP || dtype_size(t.dtype) == 0 || t.rank < 0 || t.rank > EMX_MAX_RANK)
      return set_error(EMX_ERR_PLAN_FORMAT, "tensor %zu: bad kind/dtype/rank", i);
    if (t.offset > limit || t.nbytes > limit - t.offset)
      return set_error(EMX_ERR_PLAN_FORMAT, "tensor %zu: [%llu, +%llu) outside its region (%llu bytes)", i,
                       (unsigned long long)t.offset, (unsigned long long)t.nbytes, (unsigned long long)limit);
  }
  for (uint32_t id : p->inputs)
    if (id >= h.n_tensors || p->tensors[id].kind != EMX_T_INPUT) return set_error(EMX_ERR_PLAN_FORMAT, "bad input id");
  for (uint32_t id : p->outputs)
    if (id >= h.n_tensors || p->tensors[id].kind != EMX_T_OUTPUT) return set_error(EMX_ERR_PLAN_FORMAT, "bad output id");
  p->entries.resize(h.n_ops);
  for (size_t i = 0; i < p->ops.size(); ++i) {
    const PlanOp& op = p->ops[i];
    p->entries[i] = find_kernel(op.kernel);
    if (!p->entries[i]) return set_error(EMX_ERR_UNSUPPORTED, "op %zu: unknown kernel id %u", i, op.kernel);
    if (op.n_tensors > EMX_OP_MAX_TENSORS) return set_error(EMX_ERR_PLAN_FORMAT, "op %zu: too many tensors", i);
    for (uint32_t j = 0; j < op.n_tensors; ++j)
      if (op.t[j] < -1 || op.t[j] >= (int32_t)h.n_tensors)
        return set_error(EMX_ERR_PLAN_FORMAT, "op %zu: tensor ref %d out of range", i, op.t[j]);
  }
  return EMX_OK;
}

int load_common(emx_plan* p, const void* plan, size_t plan_len, int device) {
  int rc = parse_plan(p, plan, plan_len);
  if (rc) return rc;
  int ndev = 0;
  CUDA_TRY(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return set_error(EMX_ERR_INVALID_ARGUMENT, "device %d of %d", device, ndev);
  p->device = device;
  CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  CUDA_TRY(cudaDeviceGetAttribute(&p->num_sms, cudaDevAttrMultiProcessorCount, device), "sm count");
  if (cudaMalloc(&p->d_arena, p->hdr.arena_bytes ? p->hdr.arena_bytes : 256) != cudaSuccess)
    return set_error(EMX_ERR_OUT_OF_MEMORY, "arena allocation of %llu bytes failed",
                     (unsigned long long)p->hdr.arena_bytes);
  if (cudaMalloc(&p->d_weights, p->hdr.weight_bytes ? p->hdr.weight_bytes : 256) != cudaSuccess)
    return set_error(EMX_ERR_OUT_OF_MEMORY, "weight allocation of %llu bytes failed",
                     (unsigned long long)p->hdr.weight_bytes);
  CUDA_TRY(cudaMalloc(&p->d_error, 256), "error word");
  CUDA_TRY(cudaMemset(p->d_error, 0, 256), "error word");
  // zero the arena once: zero-bordered layouts rely on borders never being written
  CUDA_TRY(cudaMemset(p->d_arena, 0, p->hdr.arena_bytes ? p->hdr.arena_bytes : 256), "arena memset");
  CUDA_TRY(cudaStreamCreateWithFlags(&p->own_stream, cudaStreamNonBlocking), "stream");
  p->ptrs.assign(p->tensors.size(), nullptr);
  for (size_t i = 0; i < p->tensors.size(); ++i) {
    const PlanTensor& t = p->tensors[i];
    uint8_t* base = static_cast<uint8_t*>(t.kind == EMX_T_WEIGHT ? p->d_weights : p->d_arena);
    p->ptrs[i] = base + t.offset;
  }
  return EMX_OK;
}

int prepare_ops(emx_plan* p) {
  p->states.resize(p->ops.size());
  for (size_t i = 0; i < p->ops.size(); ++i) {
    if (!p->entries[i]->prepare) continue;
    char msg[512] = {0};
    int rc = p->entries[i]->prepare(p->ops[i], p->ptrs.data(), &p->states[i], p->device, msg, sizeof(msg));
    if (rc) return set_error(rc, "op %zu (%s): %s", i, p->entries[i]->name, msg);
  }
  return EMX_OK;
}

void destroy(emx_plan* p) {
  if (!p) return;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(p->device);
  for (auto& g : p->graphs) cudaGraphExecDestroy(g.exec);
  if (p->h_hold) cudaFreeHost(p->h_hold);
  for (auto e : p->ev_in) cudaEventDestroy(e);
  for (auto e : p->ev_comp) cudaEventDestroy(e);
  if (p->ev_start) cudaEventDestroy(p->ev_start);
  if (p->ev_done) cudaEventDestroy(p->ev_done);
  if (p->copy_in) cudaStreamDestroy(p->copy_in);
  if (p->copy_out) cudaStreamDestroy(p->copy_out);
  if (p->d_io) cudaFree(p->d_io);
  for (int k = 0; k < 2; ++k) {
    if (p->d_io2[k]) cudaFree(p->d_io2[k]);
    if (p->ov_h2d[k]) cudaEventDestroy(p->ov_h2d[k]);
    if (p->ov_comp[k]) cudaEventDestroy(p->ov_comp[k]);
    if (p->ov_d2h[k]) cudaEventDestroy(p->ov_d2h[k]);
  }
  for (auto e : p->ev_begin) cudaEventDestroy(e);
  for (auto e : p->ev_end) cudaEventDestroy(e);
  if (p->own_stream) cudaStreamDestroy(p->own_stream);
  if (p->d_arena) cudaFree(p->d_arena);
  if (p->d_weights) cudaFree(p->d_weights);
  if (p->d_error) cudaFree(p->d_error);
  cudaSetDevice(cur);
  delete p;
}

// Enqueue every op of the plan on `stream`.  In profiling mode each op is
// bracketed by timing events and the whole sequence sits behind a hold kernel
// that spins (at most ~1 s) on a host-mapped flag until the host has
// enqueued everything, so the GPU then runs the ops back to back and the
// events measure kernels rather than host launch gaps.
int launch_ops(emx_plan* p, int64_t run_batch, cudaStream_t stream, int* launches) {
  emx::LaunchCtx ctx{stream, p->d_error, run_batch, p->num_sms};
  ctx.fault = p->fault;
  ctx.ops = p->ops.data();
  ctx.states = p->states.data();
  ctx.n_ops = p->ops.size();
  const int seq = ++p->hold_seq;
  if (p->profiling) emx::launch_hold(p->d_hold, seq, p->d_error, stream);
  for (size_t i = 0; i < p->ops.size(); ++i) {
    ctx.index = i;
    if (p->profiling) cudaEventRecord(p->ev_begin[i], stream);
    int rc = p->entries[i]->launch(p->ops[i], p->ptrs.data(), &p->states[i], ctx, launches);
    if (p->profiling) cudaEventRecord(p->ev_end[i], stream);
    if (rc) {
      if (p->profiling) *(volatile int*)p->h_hold = seq;
      cudaError_t e = cudaGetLastError();
      return set_error(rc == EMX_ERR_CUDA ? EMX_ERR_CUDA : rc, "op %zu (%s) launch failed: %s", i,
                       p->entries[i]->name, cudaGetErrorString(e));
    }
  }
  if (p->profiling) {
    __sync_synchronize();
    *(volatile int*)p->h_hold = seq;
  }
  return EMX_OK;
}

// The plan's kernels as one CUDA graph per (I/O pointers, batch, profiling):
// captured once on the plan's private stream, replayed with one
// cudaGraphLaunch on the caller's stream.  Host<->device staging copies stay
// outside the graph (they may involve pageable host memory).
int run_graph(emx_plan* p, int64_t run_batch, cudaStream_t stream, int* launches) {
  if (p->ops.empty()) return EMX_OK;  // every op had only empty outputs: nothing to launch
  std::vector<void*> key;
  key.reserve(p->inputs.size() + p->outputs.size());
  for (uint32_t id : p->inputs) key.push_back(p->ptrs[id]);
  for (uint32_t id : p->outputs) key.push_back(p->ptrs[id]);
  ++p->graph_clock;
  for (auto& g : p->graphs) {
    if (g.batch == run_batch && g.profiling == p->profiling && g.key == key) {
      g.last_use = p->graph_clock;
      *launches += g.launches;
      CUDA_TRY(cudaGraphLaunch(g.exec, stream), "cudaGraphLaunch");
      return EMX_OK;
    }
  }
  cudaGraph_t graph = nullptr;
  CUDA_TRY(cudaStreamBeginCapture(p->own_stream, cudaStreamCaptureModeThreadLocal), "begin capture");
  int n = 0;
  int rc = launch_ops(p, run_batch, p->own_stream, &n);
  cudaError_t e = cudaStreamEndCapture(p->own_stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return set_error(EMX_ERR_CUDA, "end capture: %s", cudaGetErrorString(e));
  emx_plan::GraphEntry entry;
  entry.key = key;
  entry.batch = run_batch;
  entry.profiling = p->profiling;
  entry.launches = n;
  entry.last_use = p->graph_clock;
  e = cudaGraphInstantiate(&entry.exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return set_error(EMX_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
  if (p->graphs.size() >= 8) {  // evict the least recently used
    size_t lru = 0;
    for (size_t i = 1; i < p->graphs.size(); ++i)
      if (p->graphs[i].last_use < p->graphs[lru].last_use) lru = i;
    cudaGraphExecDestroy(p->graphs[lru].exec);
    p->graphs.erase(p->graphs.begin() + lru);
  }
  p->graphs.push_back(entry);
  *launches += n;
  CUDA_TRY(cudaGraphLaunch(entry.exec, stream), "cudaGraphLaunch");
  return EMX_OK;
}

// Where a caller's buffer lives: device (or managed) memory is used in place;
// page-locked host memory can be copied asynchronously (and pipelined);
// pageable host memory is staged with ordinary copies.
enum MemKind { MEM_DEVICE = 0, MEM_PINNED = 1, MEM_PAGEABLE = 2 };

int mem_kind(const void* ptr) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();
    return MEM_PAGEABLE;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return MEM_DEVICE;
  return a.type == cudaMemoryTypeHost ? MEM_PINNED : MEM_PAGEABLE;
}

// bytes of one batch row along axis 0 (tensor must be batched)
size_t row_bytes(const PlanTensor& t) {
  if (t.rank < 1 || t.dims[0] <= 0) return 0;
  return (size_t)(t.nbytes / (uint64_t)t.dims[0]);
}

constexpr size_t kPipelineMinHostBytes = 1u << 20;

// Whether a run can split its batch into slices whose host copies overlap the
// kernels: a batchable plan, every output batched on axis 0, every host
// buffer page-locked, at least 1 MiB crossing the bus, two or more rows.
bool can_pipeline(const emx_plan* p, int64_t count) {
  if (p->io_chunks < 2 || p->profiling || count < 2 || p->hdr.batch <= 0 || !(p->hdr.flags & EMX_PLAN_BATCHABLE))
    return false;
  size_t host_bytes = 0;
  for (size_t i = 0; i < p->inputs.size(); ++i) {
    const PlanTensor& t = p->tensors[p->inputs[i]];
    if (p->in_kind[i] == MEM_DEVICE) continue;
    if (p->in_kind[i] != MEM_PINNED) return false;
    host_bytes += t.batch_axis == 0 ? (size_t)count * row_bytes(t) : (size_t)t.nbytes;
  }
  for (size_t i = 0; i < p->outputs.size(); ++i) {
    const PlanTensor& t = p->tensors[p->outputs[i]];
    if (t.batch_axis != 0 || row_bytes(t) == 0) return false;
    if (p->out_kind[i] == MEM_DEVICE) continue;
    if (p->out_kind[i] != MEM_PINNED) return false;
    host_bytes += (size_t)count * row_bytes(t);
  }
  return host_bytes >= kPipelineMinHostBytes;
}

int ensure_pipeline(emx_plan* p) {
  if (!p->copy_in) CUDA_TRY(cudaStreamCreateWithFlags(&p->copy_in, cudaStreamNonBlocking), "copy-in stream");
  if (!p->copy_out) CUDA_TRY(cudaStreamCreateWithFlags(&p->copy_out, cudaStreamNonBlocking), "copy-out stream");
  if (!p->ev_start) CUDA_TRY(cudaEventCreateWithFlags(&p->ev_start, cudaEventDisableTiming), "event");
  if (!p->ev_done) CUDA_TRY(cudaEventCreateWithFlags(&p->ev_done, cudaEventDisableTiming), "event");
  while ((int)p->ev_in.size() < p->io_chunks) {
    cudaEvent_t a = nullptr, b = nullptr;
    CUDA_TRY(cudaEventCreateWithFlags(&a, cudaEventDisableTiming), "event");
    p->ev_in.push_back(a);
    CUDA_TRY(cudaEventCreateWithFlags(&b, cudaEventDisableTiming), "event");
    p->ev_comp.push_back(b);
  }
  if (!p->d_io) {
    size_t total = 0;
    p->io_off.clear();
    for (uint32_t id : p->inputs) { p->io_off.push_back(total); total += (p->tensors[id].nbytes + 255) & ~(size_t)255; }
    for (uint32_t id : p->outputs) { p->io_off.push_back(total); total += (p->tensors[id].nbytes + 255) & ~(size_t)255; }
    if (cudaMalloc(&p->d_io, total ? total : 256) != cudaSuccess) {
      cudaGetLastError();
      return set_error(EMX_ERR_OUT_OF_MEMORY, "host I/O staging of %zu bytes failed", total);
    }
  }
  return EMX_OK;
}

// The run as `chunks` batch slices: slice i's host inputs are uploaded on
// copy_in, its kernels run on the caller's stream once they have arrived,
// and its host outputs are downloaded on copy_out once its kernels are done,
// so uploads, kernels and downloads of neighbouring slices overlap.  Slices
// stage through d_io at their own rows, never through the arena, whose
// regions later kernels reuse.  The caller's stream waits for the last
// download before the call's work is complete.
int run_pipelined(emx_plan* p, const void* const* inputs, void* const* outputs, int64_t b0, int64_t count,
                  cudaStream_t S) {
  int rc = ensure_pipeline(p);
  if (rc) return rc;
  uint8_t* io = static_cast<uint8_t*>(p->d_io);
  const size_t nin = p->inputs.size();
  CUDA_TRY(cudaEventRecord(p->ev_start, S), "event record");
  CUDA_TRY(cudaStreamWaitEvent(p->copy_in, p->ev_start, 0), "stream wait");
  CUDA_TRY(cudaStreamWaitEvent(p->copy_out, p->ev_start, 0), "stream wait");
  // inputs without a batch axis: whole, once, ahead of the first slice
  for (size_t i = 0; i < nin; ++i) {
    const uint32_t id = p->inputs[i];
    const PlanTensor& t = p->tensors[id];
    if (t.batch_axis == 0) continue;
    if (p->in_kind[i] == MEM_DEVICE) {
      p->ptrs[id] = const_cast<void*>(inputs[i]);
    } else {
      CUDA_TRY(cudaMemcpyAsync(io + p->io_off[i], inputs[i], t.nbytes, cudaMemcpyHostToDevice, p->copy_in),
               "input upload");
      p->ptrs[id] = io + p->io_off[i];
    }
  }
  const int64_t rows = (count + p->io_chunks - 1) / p->io_chunks;
  int launches = 0;
  for (int c = 0; c * rows < count; ++c) {
    const int64_t r0 = b0 + c * rows, rn = std::min<int64_t>(rows, b0 + count - r0);
    for (size_t i = 0; i < nin; ++i) {
      const uint32_t id = p->inputs[i];
      const PlanTensor& t = p->tensors[id];
      if (t.batch_axis != 0) continue;
      const size_t rb = row_bytes(t), off = (size_t)r0 * rb;
      if (p->in_kind[i] == MEM_DEVICE) {
        p->ptrs[id] = const_cast<uint8_t*>(static_cast<const uint8_t*>(inputs[i]) + off);
      } else {
        uint8_t* dst = io + p->io_off[i] + off;
        CUDA_TRY(cudaMemcpyAsync(dst, static_cast<const uint8_t*>(inputs[i]) + off, (size_t)rn * rb,
                                 cudaMemcpyHostToDevice, p->copy_in), "input upload");
        p->ptrs[id] = dst;
      }
    }
    CUDA_TRY(cudaEventRecord(p->ev_in[c], p->copy_in), "event record");
    CUDA_TRY(cudaStreamWaitEvent(S, p->ev_in[c], 0), "stream wait");
    for (size_t i = 0; i < p->outputs.size(); ++i) {
      const uint32_t id = p->outputs[i];
      const size_t off = (size_t)r0 * row_bytes(p->tensors[id]);
      p->ptrs[id] = p->out_kind[i] == MEM_DEVICE ? static_cast<uint8_t*>(outputs[i]) + off
                                                   : io + p->io_off[nin + i] + off;
    }
    rc = p->use_graphs ? run_graph(p, rn, S, &launches) : launch_ops(p, rn, S, &launches);
    if (rc) return rc;
    CUDA_TRY(cudaEventRecord(p->ev_comp[c], S), "event record");
    CUDA_TRY(cudaStreamWaitEvent(p->copy_out, p->ev_comp[c], 0), "stream wait");
    for (size_t i = 0; i < p->outputs.size(); ++i) {
      if (p->out_kind[i] == MEM_DEVICE) continue;
      const uint32_t id = p->outputs[i];
      const size_t rb = row_bytes(p->tensors[id]), off = (size_t)r0 * rb;
      CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(outputs[i]) + off, io + p->io_off[nin + i] + off,
                               (size_t)rn * rb, cudaMemcpyDeviceToHost, p->copy_out), "output download");
    }
  }
  CUDA_TRY(cudaEventRecord(p->ev_done, p->copy_out), "event record");
  CUDA_TRY(cudaStreamWaitEvent(S, p->ev_done, 0), "stream wait");
  p->launches_total += launches;
  p->launches_last = launches;
  p->events_pending = false;
  return EMX_OK;
}

// Overlapped runs need every host buffer page-locked (device buffers are used in place).
bool can_overlap(const emx_plan* p) {
  if (!p->io_overlap || p->profiling) return false;
  bool any_host = false;
  for (int k : p->in_kind) {
    if (k == MEM_PAGEABLE) return false;
    any_host = any_host || k == MEM_PINNED;
  }
  for (int k : p->out_kind) {
    if (k == MEM_PAGEABLE) return false;
    any_host = any_host || k == MEM_PINNED;
  }
  return any_host;
}

int ensure_overlap(emx_plan* p) {
  if (!p->copy_in) CUDA_TRY(cudaStreamCreateWithFlags(&p->copy_in, cudaStreamNonBlocking), "copy-in stream");
  if (!p->copy_out) CUDA_TRY(cudaStreamCreateWithFlags(&p->copy_out, cudaStreamNonBlocking), "copy-out stream");
  if (p->io_off.empty()) {
    size_t total = 0;
    for (uint32_t id : p->inputs) { p->io_off.push_back(total); total += (p->tensors[id].nbytes + 255) & ~(size_t)255; }
    for (uint32_t id : p->outputs) { p->io_off.push_back(total); total += (p->tensors[id].nbytes + 255) & ~(size_t)255; }
  }
  size_t total = 0;
  for (size_t i = 0; i < p->inputs.size(); ++i) total = p->io_off[i] + ((p->tensors[p->inputs[i]].nbytes + 255) & ~(size_t)255);
  for (size_t i = 0; i < p->outputs.size(); ++i)
    total = std::max(total, p->io_off[p->inputs.size() + i] + ((p->tensors[p->outputs[i]].nbytes + 255) & ~(size_t)255));
  for (int k = 0; k < 2; ++k) {
    if (!p->d_io2[k] && cudaMalloc(&p->d_io2[k], total ? total : 256) != cudaSuccess) {
      cudaGetLastError();
      return set_error(EMX_ERR_OUT_OF_MEMORY, "overlapped host I/O staging of 2 x %zu bytes failed", total);
    }
    if (!p->ov_h2d[k]) CUDA_TRY(cudaEventCreateWithFlags(&p->ov_h2d[k], cudaEventDisableTiming), "event");
    if (!p->ov_comp[k]) CUDA_TRY(cudaEventCreateWithFlags(&p->ov_comp[k], cudaEventDisableTiming), "event");
    if (!p->ov_d2h[k]) CUDA_TRY(cudaEventCreateWithFlags(&p->ov_d2h[k], cudaEventDisableTiming), "event");
  }
  return EMX_OK;
}

// One overlapped run on staging set k = run number % 2: the upload (copy_in)
// waits only until the run two back has finished reading set k's inputs, the
// kernels (caller's stream) wait for their upload, for the previous run's
// kernels (the arena is shared) and for set k's previous download, and the
// download (copy_out) waits for the kernels.  The caller's stream is not made
// to wait for the download: emx_b200_join / emx_b200_sync do that.
int run_overlapped(emx_plan* p, const void* const* inputs, void* const* outputs, int64_t b0, int64_t count,
                   cudaStream_t S) {
  int rc = ensure_overlap(p);
  if (rc) return rc;
  const int k = (int)(p->ov_seq & 1u);
  const bool have_prev = p->ov_seq > 0, have_two_back = p->ov_seq > 1;
  ++p->ov_seq;
  uint8_t* io = static_cast<uint8_t*>(p->d_io2[k]);
  const size_t nin = p->inputs.size();
  const int64_t full = p->hdr.batch;
  if (have_two_back) CUDA_TRY(cudaStreamWaitEvent(p->copy_in, p->ov_comp[k], 0), "stream wait");
  for (size_t i = 0; i < nin; ++i) {
    const uint32_t id = p->inputs[i];
    const PlanTensor& t = p->tensors[id];
    size_t off = 0, bytes = t.nbytes;
    if (full > 0 && t.batch_axis == 0) {
      off = (size_t)b0 * row_bytes(t);
      bytes = (size_t)count * row_bytes(t);
    }
    if (p->in_kind[i] == MEM_DEVICE) {
      p->ptrs[id] = const_cast<uint8_t*>(static_cast<const uint8_t*>(inputs[i]) + off);
    } else {
      CUDA_TRY(cudaMemcpyAsync(io + p->io_off[i], static_cast<const uint8_t*>(inputs[i]) + off, bytes,
                               cudaMemcpyHostToDevice, p->copy_in), "input upload");
      p->ptrs[id] = io + p->io_off[i];
    }
  }
  CUDA_TRY(cudaEventRecord(p->ov_h2d[k], p->copy_in), "event record");
  CUDA_TRY(cudaStreamWaitEvent(S, p->ov_h2d[k], 0), "stream wait");
  if (have_prev) CUDA_TRY(cudaStreamWaitEvent(S, p->ov_comp[k ^ 1], 0), "stream wait");
  if (have_two_back) CUDA_TRY(cudaStreamWaitEvent(S, p->ov_d2h[k], 0), "stream wait");
  for (size_t i = 0; i < p->outputs.size(); ++i) {
    const uint32_t id = p->outputs[i];
    const PlanTensor& t = p->tensors[id];
    const size_t off = (full > 0 && t.batch_axis == 0) ? (size_t)b0 * row_bytes(t) : 0;
    p->ptrs[id] = p->out_kind[i] == MEM_DEVICE ? static_cast<uint8_t*>(outputs[i]) + off : io + p->io_off[nin + i];
  }
  int launches = 0;
  const int64_t run_batch = full > 0 ? count : 0;
  rc = p->use_graphs ? run_graph(p, run_batch, S, &launches) : launch_ops(p, run_batch, S, &launches);
  if (rc) return rc;
  CUDA_TRY(cudaEventRecord(p->ov_comp[k], S), "event record");
  CUDA_TRY(cudaStreamWaitEvent(p->copy_out, p->ov_comp[k], 0), "stream wait");
  for (size_t i = 0; i < p->outputs.size(); ++i) {
    if (p->out_kind[i] == MEM_DEVICE) continue;
    const PlanTensor& t = p->tensors[p->outputs[i]];
    size_t off = 0, bytes = t.nbytes;
    if (full > 0 && t.batch_axis == 0) {
      off = (size_t)b0 * row_bytes(t);
      bytes = (size_t)count * row_bytes(t);
    }
    CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(outputs[i]) + off, io + p->io_off[nin + i], bytes,
                             cudaMemcpyDeviceToHost, p->copy_out), "output download");
  }
  CUDA_TRY(cudaEventRecord(p->ov_d2h[k], p->copy_out), "event record");
  p->ov_last = p->ov_d2h[k];
  p->launches_total += launches;
  p->launches_last = launches;
  p->events_pending = false;
  return EMX_OK;
}

}  // namespace

extern "C" {

const char* emx_b200_version(void) { return "0.1.0"; }

const char* emx_b200_last_error(void) { return g_last_error.c_str(); }

int emx_b200_plan_load_mem(const void* plan, size_t plan_len, const void* weights, size_t weights_len, int device,
                           emx_plan_t** out) {
  if (!out) return set_error(EMX_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  emx_plan* p = new emx_plan();
  int rc = load_common(p, plan, plan_len, device);
  if (!rc && weights_len != p->hdr.weight_bytes)
    rc = set_error(EMX_ERR_WEIGHTS, "weight blob is %zu bytes, plan expects %llu", weights_len,
                   (unsigned long long)p->hdr.weight_bytes);
  if (!rc && weights_len) {
    if (!weights) rc = set_error(EMX_ERR_INVALID_ARGUMENT, "weights is NULL");
    else if (cudaMemcpy(p->d_weights, weights, weights_len, cudaMemcpyHostToDevice) != cudaSuccess)
      rc = set_error(EMX_ERR_CUDA, "weight upload failed");
  }
  if (!rc) rc = prepare_ops(p);
  if (rc) {
    destroy(p);
    return rc;
  }
  g_last_error.clear();
  *out = p;
  return EMX_OK;
}

int emx_b200_plan_load(const void* plan, size_t plan_len, const char* weights_path, int device, emx_plan_t** out) {
  if (!out) return set_error(EMX_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  if (plan_len < sizeof(PlanHeader) || !plan) return set_error(EMX_ERR_PLAN_FORMAT, "plan blob too short");
  PlanHeader h;
  memcpy(&h, plan, sizeof(h));
  std::vector<uint8_t> buf;
  if (h.weight_bytes) {
    if (!weights_path) return set_error(EMX_ERR_WEIGHTS, "plan has %llu weight bytes but no weights path",
                                        (unsigned long long)h.weight_bytes);
    FILE* f = fopen(weights_path, "rb");
    if (!f) return set_error(EMX_ERR_WEIGHTS, "cannot open weights file '%s'", weights_path);
    buf.resize(h.weight_bytes);
    size_t got = fread(buf.data(), 1, buf.size(), f);
    int extra = fgetc(f);
    fclose(f);
    if (got != buf.size())
      return set_error(EMX_ERR_WEIGHTS, "weights file '%s': short read (%zu of %llu bytes)", weights_path, got,
                       (unsigned long long)h.weight_bytes);
    if (extra != EOF) return set_error(EMX_ERR_WEIGHTS, "weights file '%s' is longer than the plan expects", weights_path);
  }
  return emx_b200_plan_load_mem(plan, plan_len, buf.data(), buf.size(), device, out);
}

int emx_b200_run(emx_plan_t* p, const void* const* inputs, void* const* outputs, int64_t batch_begin,
                 int64_t batch_count, void* stream_) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  if ((p->inputs.size() && !inputs) || (p->outputs.size() && !outputs))
    return set_error(EMX_ERR_INVALID_ARGUMENT, "inputs/outputs array is NULL");
  const int64_t full = p->hdr.batch;
  if (batch_count < 0) batch_count = full;
  if (batch_begin < 0 || batch_count < 0 || (full > 0 && batch_begin + batch_count > full))
    return set_error(EMX_ERR_INVALID_ARGUMENT, "batch range [%lld, +%lld) outside [0, %lld)", (long long)batch_begin,
                     (long long)batch_count, (long long)full);
  const bool sliced = full > 0 && (batch_begin != 0 || batch_count != full);
  if (sliced && !(p->hdr.flags & EMX_PLAN_BATCHABLE))
    return set_error(EMX_ERR_INVALID_ARGUMENT, "this plan cannot run a batch slice (batch axis is not axis 0)");
  if (full > 0 && batch_count == 0) return EMX_OK;
  CUDA_TRY(cudaSetDevice(p->device), "cudaSetDevice");
  cudaStream_t stream = stream_ ? static_cast<cudaStream_t>(stream_) : p->own_stream;
  p->last_stream = stream;
  p->pending.clear();
  for (size_t i = 0; i < p->inputs.size(); ++i)
    if (!inputs[i]) return set_error(EMX_ERR_INVALID_ARGUMENT, "input %zu is NULL", i);
  for (size_t i = 0; i < p->outputs.size(); ++i)
    if (!outputs[i]) return set_error(EMX_ERR_INVALID_ARGUMENT, "output %zu is NULL", i);
  p->in_kind.resize(p->inputs.size());
  p->out_kind.resize(p->outputs.size());
  for (size_t i = 0; i < p->inputs.size(); ++i) p->in_kind[i] = mem_kind(inputs[i]);
  for (size_t i = 0; i < p->outputs.size(); ++i) p->out_kind[i] = mem_kind(outputs[i]);
  if (can_overlap(p)) return run_overlapped(p, inputs, outputs, batch_begin, batch_count, stream);
  if (full > 0 && can_pipeline(p, batch_count))
    return run_pipelined(p, inputs, outputs, batch_begin, batch_count, stream);
  for (size_t i = 0; i < p->inputs.size(); ++i) {
    const PlanTensor& t = p->tensors[p->inputs[i]];
    const void* src = inputs[i];
    if (!src) return set_error(EMX_ERR_INVALID_ARGUMENT, "input %zu is NULL", i);
    size_t off = 0, bytes = t.nbytes;
    if (full > 0 && t.batch_axis == 0) {
      off = (size_t)batch_begin * row_bytes(t);
      bytes = (size_t)batch_count * row_bytes(t);
    }
    void* staging = static_cast<uint8_t*>(p->d_arena) + t.offset;
    if (p->in_kind[i] == MEM_DEVICE) {
      p->ptrs[p->inputs[i]] = const_cast<uint8_t*>(static_cast<const uint8_t*>(src) + off);
    } else {
      CUDA_TRY(cudaMemcpyAsync(staging, static_cast<const uint8_t*>(src) + off, bytes, cudaMemcpyHostToDevice, stream),
               "input upload");
      p->ptrs[p->inputs[i]] = staging;
    }
  }
  for (size_t i = 0; i < p->outputs.size(); ++i) {
    const PlanTensor& t = p->tensors[p->outputs[i]];
    void* dst = outputs[i];
    if (!dst) return set_error(EMX_ERR_INVALID_ARGUMENT, "output %zu is NULL", i);
    size_t off = 0, bytes = t.nbytes;
    if (full > 0 && t.batch_axis == 0) {
      off = (size_t)batch_begin * row_bytes(t);
      bytes = (size_t)batch_count * row_bytes(t);
    }
    void* staging = static_cast<uint8_t*>(p->d_arena) + t.offset;
    if (p->out_kind[i] == MEM_DEVICE) {
      p->ptrs[p->outputs[i]] = static_cast<uint8_t*>(dst) + off;
    } else {
      p->ptrs[p->outputs[i]] = staging;
      p->pending.push_back({static_cast<uint8_t*>(dst) + off, staging, bytes});
    }
  }
  const int64_t run_batch = full > 0 ? batch_count : 0;
  int launches = 0;
  if (p->use_graphs && !p->profiling) {
    int rc = run_graph(p, run_batch, stream, &launches);
    if (rc) return rc;
  } else {
    int rc = launch_ops(p, run_batch, stream, &launches);
    if (rc) return rc;
  }
  for (const auto& pd : p->pending)
    CUDA_TRY(cudaMemcpyAsync(pd.host, pd.dev, pd.bytes, cudaMemcpyDeviceToHost, stream), "output download");
  p->launches_total += launches;
  p->launches_last = launches;
  p->events_pending = p->profiling;
  return EMX_OK;
}

int emx_b200_sync(emx_plan_t* p) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  CUDA_TRY(cudaSetDevice(p->device), "cudaSetDevice");
  CUDA_TRY(cudaStreamSynchronize(p->last_stream ? p->last_stream : p->own_stream), "stream synchronize");
  if (p->copy_in) CUDA_TRY(cudaStreamSynchronize(p->copy_in), "stream synchronize");
  if (p->copy_out) CUDA_TRY(cudaStreamSynchronize(p->copy_out), "stream synchronize");
  if (p->events_pending) {
    for (size_t i = 0; i < p->ops.size(); ++i) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, p->ev_begin[i], p->ev_end[i]) == cudaSuccess) p->op_ms[i] += ms;
    }
    ++p->profiled_runs;
    p->events_pending = false;
  }
  int err = 0;
  CUDA_TRY(cudaMemcpy(&err, p->d_error, sizeof(int), cudaMemcpyDeviceToHost), "error word read");
  if (err) {
    cudaMemset(p->d_error, 0, sizeof(int));
    return set_error(EMX_ERR_DEVICE_TIMEOUT, "device-side wait gave up (code %d)", err);
  }
  return EMX_OK;
}

void emx_b200_plan_free(emx_plan_t* p) { destroy(p); }

int emx_b200_plan_info(const emx_plan_t* p, emx_plan_info_t* info) {
  if (!p || !info) return set_error(EMX_ERR_INVALID_ARGUMENT, "NULL argument");
  info->device = p->device;
  info->n_inputs = (int32_t)p->inputs.size();
  info->n_outputs = (int32_t)p->outputs.size();
  info->n_ops = (int32_t)p->ops.size();
  info->batch = p->hdr.batch;
  info->arena_bytes = (int64_t)p->hdr.arena_bytes;
  info->weight_bytes = (int64_t)p->hdr.weight_bytes;
  info->launches_per_run = p->launches_last;
  return EMX_OK;
}

int64_t emx_b200_launch_count(const emx_plan_t* p) { return p ? p->launches_total : -1; }

int emx_b200_set_graphs(emx_plan_t* p, int enable) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  p->use_graphs = enable != 0;
  return EMX_OK;
}

int emx_b200_set_wait_budget(emx_plan_t* p, uint64_t ns) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  CUDA_TRY(cudaSetDevice(p->device), "cudaSetDevice");
  // the word 8 bytes after the error word (tc100.cuh wait_budget_ns); ordered
  // after every run already enqueued on the plan's streams
  CUDA_TRY(cudaDeviceSynchronize(), "device synchronize");
  const unsigned long long v = ns;
  CUDA_TRY(cudaMemcpy(reinterpret_cast<char*>(p->d_error) + 8, &v, sizeof(v), cudaMemcpyHostToDevice),
           "wait budget");
  return EMX_OK;
}

int emx_b200_set_fault(emx_plan_t* p, int hooks) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (hooks & ~emx::FAULT_DROP_CHAIN_PROGRESS) return set_error(EMX_ERR_INVALID_ARGUMENT, "unknown hook bits %d", hooks);
  if (hooks == p->fault) return EMX_OK;
  CUDA_TRY(cudaSetDevice(p->device), "cudaSetDevice");
  CUDA_TRY(cudaDeviceSynchronize(), "device synchronize");
  for (auto& g : p->graphs) cudaGraphExecDestroy(g.exec);  // captured with the previous hooks
  p->graphs.clear();
  p->fault = hooks;
  return EMX_OK;
}

int emx_b200_set_host_io_overlap(emx_plan_t* p, int enable) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  p->io_overlap = enable != 0;
  return EMX_OK;
}

int emx_b200_join(emx_plan_t* p, void* stream_) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  CUDA_TRY(cudaSetDevice(p->device), "cudaSetDevice");
  cudaStream_t stream = stream_ ? static_cast<cudaStream_t>(stream_) : p->own_stream;
  if (p->ov_last) CUDA_TRY(cudaStreamWaitEvent(stream, p->ov_last, 0), "stream wait");
  return EMX_OK;
}

int emx_b200_set_host_io_chunks(emx_plan_t* p, int chunks) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (chunks < 1 || chunks > 64) return set_error(EMX_ERR_INVALID_ARGUMENT, "host I/O chunks %d not in [1, 64]", chunks);
  p->io_chunks = chunks;
  return EMX_OK;
}

int emx_b200_set_profiling(emx_plan_t* p, int enable) {
  if (!p) return set_error(EMX_ERR_INVALID_ARGUMENT, "plan is NULL");
  CUDA_TRY(cudaSetDevice(p->device), "cudaSetDevice");
  if (enable && !p->h_hold) {
    CUDA_TRY(cudaHostAlloc((void**)&p->h_hold, sizeof(int), cudaHostAllocMapped), "hold flag");
    *p->h_hold = 0;
    p->hold_seq = 0;
    CUDA_TRY(cudaHostGetDevicePointer((void**)&p->d_hold, p->h_hold, 0), "hold flag device pointer");
  }
  if (enable && p->ev_begin.empty()) {
    p->ev_begin.resize(p->ops.size());
    p->ev_end.resize(p->ops.size());
    for (size_t i = 0; i < p->ops.size(); ++i) {
      CUDA_TRY(cudaEventCreate(&p->ev_begin[i]), "event");
      CUDA_TRY(cudaEventCreate(&p->ev_end[i]), "event");
    }
  }
  p->profiling = enable != 0;
  p->op_ms.assign(p->ops.size(), 0.0);
  p->profiled_runs = 0;
  p->events_pending = false;
  return EMX_OK;
}

int emx_b200_op_times(const emx_plan_t* p, double* ms, int32_t n_ops, int64_t* runs) {
  if (!p || !ms || n_ops < (int32_t)p->ops.size()) return set_error(EMX_ERR_INVALID_ARGUMENT, "bad arguments");
  for (size_t i = 0; i < p->ops.size(); ++i) ms[i] = i < p->op_ms.size() ? p->op_ms[i] : 0.0;
  if (runs) *runs = p->profiled_runs;
  return EMX_OK;
}

}  // extern "C"
