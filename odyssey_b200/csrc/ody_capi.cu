// ody_capi.cu -- host side of libodyssey_mp.so: the extern "C" ABI declared in
// include/odyssey_mp.h, the step context (device arenas, chunk tables,
// stream, NCCL communicator) and the stateless single-op entry points.
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <string>
#include <vector>

#include "../../include/odyssey_mp.h"
#include "ody_internal.h"

using namespace ody;

static thread_local std::string g_err;

static int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define ODY_CUDA(call)                                                              \
  do {                                                                              \
    cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess)                                                          \
      return fail(ODY_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// ---------------------------------------------------------------------------
// NCCL, bound at run time (dlopen) so that a process which already loaded a
// libnccl.so.2 (e.g. PyTorch's) shares it, and a single-GPU user needs none.
// ---------------------------------------------------------------------------
struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*groupStart)() = nullptr;
  ncclResult_t (*groupEnd)() = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
};

static NcclApi* nccl_api(std::string& why) {
  static NcclApi api;
  static bool tried = false;
  if (api.h) return &api;
  if (tried) {
    why = "libnccl.so.2 could not be loaded";
    return nullptr;
  }
  tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    why = std::string("dlopen libnccl.so.2: ") + dlerror();
    return nullptr;
  }
  api.getUniqueId = (decltype(api.getUniqueId))dlsym(h, "ncclGetUniqueId");
  api.commInitRankConfig = (decltype(api.commInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
  api.allGather = (decltype(api.allGather))dlsym(h, "ncclAllGather");
  api.broadcast = (decltype(api.broadcast))dlsym(h, "ncclBroadcast");
  api.groupStart = (decltype(api.groupStart))dlsym(h, "ncclGroupStart");
  api.groupEnd = (decltype(api.groupEnd))dlsym(h, "ncclGroupEnd");
  api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
  api.commAbort = (decltype(api.commAbort))dlsym(h, "ncclCommAbort");
  api.commGetAsyncError = (decltype(api.commGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
  api.getErrorString = (decltype(api.getErrorString))dlsym(h, "ncclGetErrorString");
  if (!api.getUniqueId || !api.commInitRankConfig || !api.allGather || !api.broadcast || !api.groupStart ||
      !api.groupEnd || !api.commDestroy ||
      !api.commAbort || !api.commGetAsyncError || !api.getErrorString) {
    why = "libnccl.so.2 lacks a required symbol";
    return nullptr;
  }
  api.h = h;
  return &api;
}

// ---------------------------------------------------------------------------
// The context.
// ---------------------------------------------------------------------------
struct TensorSpec {
  int64_t numel;
  int32_t gdt;
  int32_t quant;
};

struct ody_ctx {
  ody_config cfg;
  std::vector<TensorSpec> specs;
  bool finalized = false;
  bool broken = false;
  int world = 1, rank = 0;
  int gdt = -1;
  std::vector<int32_t> owner;      // global index -> rank
  std::vector<int32_t> local_of;   // global index -> local index or -1
  std::vector<TensorDesc> tdesc;   // local tensors
  std::vector<Chunk> chunks_upd;
  // layout of the gathered quantised model: every tensor's region in global
  // order (the same region sizes as the local arenas), and each rank's slice
  std::vector<int64_t> gq_off;      // per global tensor
  std::vector<int64_t> rank_qbeg, rank_qend;   // per rank, bytes
  std::vector<int32_t> rank_tbeg, rank_tend;   // per rank, tensor indices
  int64_t gq_total = 0;
  std::vector<uint32_t> jobs;  // apply-kernel job list (bit 31: requant job)
  unsigned long long wait_ns = kWaitLimitNs;  // bound on the apply kernel's readiness wait
  int64_t n_total = 0, q_total = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t done = nullptr;
  // device memory
  float *master = nullptr, *s1 = nullptr, *s2 = nullptr;
  void* grad = nullptr;
  uint8_t* qout = nullptr;
  float* qscale = nullptr;
  uint32_t* amax = nullptr;
  Chunk* d_chunks_upd = nullptr;
  uint32_t* d_jobs = nullptr;
  uint32_t* sync = nullptr;  // job ticket + per-tensor done counts
  TensorDesc* d_tdesc = nullptr;
  StatsPartial* partials = nullptr;
  unsigned* ticket = nullptr;
  DevScaler* scaler = nullptr;
  Decision* dec = nullptr;
  double* local_stats = nullptr;
  double* gathered = nullptr;
  Decision* h_dec = nullptr;  // pinned
  int grid_stats = 0, grid_apply = 0;
  bool pending = false;
  ncclComm_t comm = nullptr;
  std::string err;
  // per-pass timing: a ring of event slots, 5 events per step
  bool timing = false;
  std::vector<cudaEvent_t> tev;
  std::vector<int64_t> tpending;  // ring slots recorded but not yet read
  int64_t tnext = 0, tsteps = 0;
  double tms[4] = {0, 0, 0, 0};
  // data-parallel gradients (ody_ctx_dp_attach): the full-model gradient
  // buffer, each tensor's offset in it, the ranks' buffers as mapped here
  bool dp_on = false;
  void* dp_buf = nullptr;
  int64_t dp_total = 0, dp_shard_off = 0;
  std::vector<int64_t> dp_off;
  std::vector<void*> dp_opened;  // peers' buffers opened through CUDA IPC
  const void** d_peers = nullptr;
  double* bar_send = nullptr;
  double* bar_recv = nullptr;
  // graph mode: the captured step and its apply-kernel node
  bool graph_mode = false;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t gexec = nullptr;
  cudaGraphNode_t gapply = nullptr;
  OptConsts goc;
  // double-buffered gradients (ody_ctx_set_grad_double_buffer): uploads of
  // step t+1's gradients into one arena on a copy stream while step t reads
  // the other; grad_slot[0] is `grad`
  bool dbuf = false;
  void* grad_slot[2] = {nullptr, nullptr};
  int upload_slot = 0;                 // the arena ODY_BUF_GRAD names (the next step reads it)
  cudaStream_t copy_stream = nullptr;  // non-blocking
  cudaEvent_t slot_read[2] = {nullptr, nullptr};  // last step reading the slot is done with it
  cudaEvent_t slot_filled[2] = {nullptr, nullptr};  // uploads into the slot are done
  bool slot_ordered = false;  // the copy stream already waits for the upload slot's last reader
};

// the gradient arena the next step reads
static void* step_grad(const ody_ctx* c) { return c->dbuf ? c->grad_slot[c->upload_slot] : c->grad; }

static constexpr int kTimingRing = 64;

static cudaError_t timing_collect(ody_ctx* c, int64_t slot) {
  cudaEvent_t* e = &c->tev[(size_t)(slot % kTimingRing) * 5];
  cudaError_t r = cudaEventSynchronize(e[4]);
  if (r != cudaSuccess) return r;
  for (int k = 0; k < 4; k++) {
    float ms = 0.0f;
    r = cudaEventElapsedTime(&ms, e[k], e[k + 1]);
    if (r != cudaSuccess) return r;
    c->tms[k] += ms;
  }
  c->tsteps += 1;
  return cudaSuccess;
}

static bool is_device_ptr(const void* p);  // device memory of the current GPU, or managed

static int ctx_fail(ody_ctx* c, int code, const std::string& msg) {
  g_err = msg;
  if (c) c->err = msg;
  return code;
}

static size_t dtype_size(int gdt) { return gdt == DT_F32 ? 4 : 2; }

extern "C" int ody_abi_version(void) { return ODY_ABI_VERSION; }

extern "C" const char* ody_last_error(const ody_ctx* ctx) {
  if (ctx && !ctx->err.empty()) return ctx->err.c_str();
  return g_err.c_str();
}

extern "C" void ody_config_default(ody_config* c) {
  memset(c, 0, sizeof(*c));
  c->optimizer = ODY_ADAMW;
  c->device = 0;
  c->learning_rate = 1e-3;
  c->momentum = 0.0;
  c->beta1 = 0.9;
  c->beta2 = 0.999;
  c->epsilon = 1e-8;
  c->weight_decay = 0.0;
  c->use_gradient_scaler = 1;
  c->initial_scale = 65536.0f;
  c->growth_factor = 2.0f;
  c->backoff_factor = 0.5f;
  c->growth_interval = 2000;
  c->min_scale = 1.0f;
  c->max_scale = 65536.0f;
  c->clip_enabled = 0;
  c->max_norm = 1.0f;
  c->comm_timeout_ms = 60000;
  c->alpha = 0.99;
}

// optimizers whose step takes a timestep t >= 1 (adam.mojo:118,
// adamw.mojo:118, rmsprop.mojo:125)
static bool needs_timestep(int opt) { return opt == ODY_ADAM || opt == ODY_ADAMW || opt == ODY_RMSPROP; }

extern "C" int64_t ody_quant_bytes(int32_t kind, int64_t n) {
  if (n < 0) return -1;
  switch (kind) {
    case ODY_Q_NONE:
      return 0;
    case ODY_Q_FP16:
    case ODY_Q_BF16:
      return 2 * n;
    case ODY_Q_FP8_E4M3:
    case ODY_Q_FP8_E5M2:
    case ODY_Q_FP8_E4M3_TENSOR:
      return n;
    case ODY_Q_MXFP4:
    case ODY_Q_MXFP4_OCP:
      return ((n + 31) / 32) * 17;
    case ODY_Q_NVFP4:
    case ODY_Q_NVFP4_TENSOR:
      return ((n + 15) / 16) * 9;
    default:
      return -1;
  }
}

// bytes of a tensor's region in the quantised-output arena: whole tiles
static int64_t quant_region(int kind, int64_t npad) {
  const int64_t tiles = (npad + kTile - 1) / kTile;
  int64_t b = 0;
  switch (kind) {
    case Q_FP16:
    case Q_BF16:
      b = 2 * npad;
      break;
    case Q_FP8_E4M3:
    case Q_FP8_E5M2:
    case Q_FP8_E4M3_TENSOR:
      b = npad;
      break;
    case Q_MXFP4:
      b = tiles * kMxTileBytes;
      break;
    case Q_NVFP4:
    case Q_NVFP4_TENSOR:
      b = tiles * kNvTileBytes;
      break;
    default:
      b = 0;
  }
  return (b + 255) / 256 * 256;
}

extern "C" int ody_ctx_create(ody_ctx** out, const ody_config* cfg) {
  if (!out || !cfg) return fail(ODY_ERR_ARG, "ody_ctx_create: null argument");
  if (cfg->optimizer < ODY_SGD || cfg->optimizer > ODY_ADAGRAD)
    return fail(ODY_ERR_ARG, "unknown optimizer " + std::to_string(cfg->optimizer));
  if (cfg->clip_enabled && !(cfg->max_norm > 0.0f))
    return fail(ODY_ERR_ARG, "max_norm must be positive, got: " + std::to_string(cfg->max_norm));
  if (cfg->use_gradient_scaler && cfg->initial_scale == 0.0f)
    return fail(ODY_ERR_ARG, "Cannot unscale with zero scale factor");
  if (cfg->chunk_elems < 0 || cfg->chunk_elems % kTile != 0 || cfg->chunk_elems > kChunk)
    return fail(ODY_ERR_ARG, "chunk_elems must be 0 or a multiple of " + std::to_string(kTile) + " up to " +
                                 std::to_string(kChunk));
  if (cfg->requant_placement < ODY_REQUANT_AUTO || cfg->requant_placement > ODY_REQUANT_AT_END)
    return fail(ODY_ERR_ARG, "unknown requant_placement " + std::to_string(cfg->requant_placement));
  ody_ctx* c = new ody_ctx();
  c->cfg = *cfg;
  if (c->cfg.comm_timeout_ms <= 0) c->cfg.comm_timeout_ms = 60000;
  *out = c;
  return ODY_OK;
}

extern "C" int ody_ctx_add_tensor(ody_ctx* c, int64_t numel, int32_t gdt, int32_t quant, int32_t* idx) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context already finalized");
  if (numel <= 0) return ctx_fail(c, ODY_ERR_SHAPE, "Cannot unscale empty gradient tensor");
  if (gdt < DT_F32 || gdt > DT_BF16) return ctx_fail(c, ODY_ERR_DTYPE, "unsupported gradient dtype");
  if (quant < ODY_Q_NONE || quant > ODY_Q_NVFP4_TENSOR)
    return ctx_fail(c, ODY_ERR_ARG, "unknown quantisation kind " + std::to_string(quant));
  if (c->gdt >= 0 && c->gdt != gdt)
    return ctx_fail(c, ODY_ERR_DTYPE, "all tensors of a context must share one gradient dtype");
  c->gdt = gdt;
  c->specs.push_back({numel, gdt, quant});
  if (idx) *idx = (int32_t)c->specs.size() - 1;
  return ODY_OK;
}

extern "C" int ody_plan_shards(const int64_t* numels, int32_t nt, int32_t world, int32_t* owner) {
  if (!numels || !owner || nt < 0 || world < 1) return fail(ODY_ERR_ARG, "ody_plan_shards: bad argument");
  // Contiguous groups of whole tensors; rank r takes tensors until the
  // running total passes (r+1)/world of all elements (closest boundary).
  double total = 0;
  for (int i = 0; i < nt; i++) total += (double)numels[i];
  double run = 0;
  int r = 0;
  for (int i = 0; i < nt; i++) {
    // move to the next rank when this tensor's midpoint lies past the
    // current rank's share of the running total
    while (r < world - 1 && run + 0.5 * (double)numels[i] > total * (r + 1) / world) r++;
    owner[i] = r;
    run += (double)numels[i];
  }
  // every rank keeps at least its order; ranks may own nothing when there
  // are fewer tensors than ranks
  return ODY_OK;
}

extern "C" int ody_nccl_unique_id(void* out128) {
  if (!out128) return fail(ODY_ERR_ARG, "null output");
  std::string why;
  NcclApi* api = nccl_api(why);
  if (!api) return fail(ODY_ERR_NCCL, why);
  ncclUniqueId id;
  ncclResult_t r = api->getUniqueId(&id);
  if (r != ncclSuccess) return fail(ODY_ERR_NCCL, std::string("ncclGetUniqueId: ") + api->getErrorString(r));
  memcpy(out128, &id, sizeof(id));
  return ODY_OK;
}

static int wait_nccl(ody_ctx* c, NcclApi* api, const char* what) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = api->commGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return ctx_fail(c, ODY_ERR_NCCL, std::string(what) + ": " + api->getErrorString(r));
    if (st == ncclSuccess) return ODY_OK;
    if (st != ncclInProgress) {
      api->commAbort(c->comm);
      c->comm = nullptr;
      c->broken = true;
      return ctx_fail(c, ODY_ERR_NCCL, std::string(what) + ": " + api->getErrorString(st));
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > c->cfg.comm_timeout_ms) {
      api->commAbort(c->comm);
      c->comm = nullptr;
      c->broken = true;
      return ctx_fail(c, ODY_ERR_COMM_TIMEOUT, std::string(what) + ": timed out after " +
                                                   std::to_string(c->cfg.comm_timeout_ms) + " ms");
    }
  }
}

template <typename T>
static cudaError_t dalloc(T** p, size_t bytes) {
  return cudaMalloc((void**)p, bytes < 256 ? 256 : bytes);
}

// Job list of the apply kernel: every update chunk, tensors in descending
// size (stable), so that the largest per-tensor-scaled tensors finish their
// updates first.  Interleaved placement (the default): the requant chunks of
// a per-tensor-scaled tensor become eligible two grid-widths of jobs after
// that tensor's last update job and are slotted in, up to two per update
// job, between the following tensors' update jobs; a tensor followed by
// fewer than two grid-widths of update jobs (the last ones of every rank)
// has its requant jobs at the end.  The decision is per tensor, so a rank of
// few large tensors (the 1B model on 4 or 8 ranks: 4,096 update jobs on a
// 592-CTA grid) still hides most of its requant work behind update traffic:
// measured 5 % faster there than all-at-end, and equal on ResNet-18.
// At-end placement: every requant job after every update job.
// nchunks[i], quant[i]: the local tensors in arena order; W: the apply grid
static std::vector<uint32_t> plan_jobs(const std::vector<int>& nchunks, const std::vector<int>& quant, size_t W,
                                       int placement) {
  std::vector<uint32_t> jobs;
  std::vector<std::pair<size_t, uint32_t>> pending;  // (eligible position, chunk)
  std::vector<uint32_t> tail;                          // requant jobs placed at the end
  size_t head = 0;
  if (W == 0) W = 1;
  const size_t nl = nchunks.size();
  std::vector<size_t> first(nl), order(nl);
  size_t total = 0;
  for (size_t li = 0; li < nl; li++) {
    first[li] = total;
    total += (size_t)nchunks[li];
    order[li] = li;
  }
  const bool interleave = placement != ODY_REQUANT_AT_END;
  const size_t delay = 2 * W;
  std::stable_sort(order.begin(), order.end(), [&](size_t x, size_t y) { return nchunks[x] > nchunks[y]; });
  size_t updates_done = 0;
  for (size_t li : order) {
    for (int k = 0; k < nchunks[li]; k++) {
      jobs.push_back((uint32_t)(first[li] + k));
      for (int r = 0; r < 2 && head < pending.size() && pending[head].first <= jobs.size(); r++)
        jobs.push_back(kRequantJob | pending[head++].second);
    }
    updates_done += (size_t)nchunks[li];
    if (quant[li] != Q_FP8_E4M3_TENSOR && quant[li] != Q_NVFP4_TENSOR) continue;
    const bool here = interleave && total - updates_done >= delay;
    for (int k = 0; k < nchunks[li]; k++) {
      if (here)
        pending.push_back({jobs.size() + delay, (uint32_t)(first[li] + k)});
      else
        tail.push_back((uint32_t)(first[li] + k));
    }
  }
  while (head < pending.size()) jobs.push_back(kRequantJob | pending[head++].second);
  for (uint32_t ch : tail) jobs.push_back(kRequantJob | ch);
  return jobs;
}

static void build_jobs(ody_ctx* c) {
  std::vector<int> nchunks, quant;
  for (const TensorDesc& d : c->tdesc) {
    nchunks.push_back(d.nchunks);
    quant.push_back(d.quant);
  }
  c->jobs = plan_jobs(nchunks, quant, (size_t)(c->grid_apply > 0 ? c->grid_apply : 1), c->cfg.requant_placement);
}

// (re)allocates the device copy of the job list and copies it in
static int upload_jobs(ody_ctx* c) {
  if (c->d_jobs) ODY_CUDA(cudaFree(c->d_jobs));
  c->d_jobs = nullptr;
  ODY_CUDA(dalloc(&c->d_jobs, sizeof(uint32_t) * (c->jobs.size() + 1)));
  if (!c->jobs.empty())
    ODY_CUDA(cudaMemcpyAsync(c->d_jobs, c->jobs.data(), sizeof(uint32_t) * c->jobs.size(), cudaMemcpyHostToDevice,
                             c->stream));
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  return ODY_OK;
}

// Test hook (not part of include/odyssey_mp.h): the apply kernel's job list
// for tensors of nchunks[i] chunks and kind quant[i] on a grid of W CTAs
// under a requant placement (ODY_REQUANT_*); jobs_out (capacity cap)
// receives the list, *njobs its length.
extern "C" int odyx_plan_jobs(const int32_t* nchunks, const int32_t* quant, int32_t nt, int32_t W,
                              int32_t placement, uint32_t* jobs_out, int64_t cap, int64_t* njobs) {
  if (nt < 0 || (nt > 0 && (!nchunks || !quant)) || !njobs) return fail(ODY_ERR_ARG, "bad argument");
  const std::vector<uint32_t> jobs = plan_jobs(std::vector<int>(nchunks, nchunks + nt),
                                               std::vector<int>(quant, quant + nt), (size_t)W, placement);
  *njobs = (int64_t)jobs.size();
  if (jobs_out) {
    if (cap < (int64_t)jobs.size()) return fail(ODY_ERR_ARG, "job buffer too small");
    std::copy(jobs.begin(), jobs.end(), jobs_out);
  }
  return ODY_OK;
}

// Test hook: the live context's apply-kernel job list and grid (the list
// ody_step runs); jobs_out may be NULL to query the length.
extern "C" int odyx_ctx_jobs(const ody_ctx* c, uint32_t* jobs_out, int64_t cap, int64_t* njobs, int32_t* grid) {
  if (!c || !njobs) return fail(ODY_ERR_ARG, "bad argument");
  if (!c->finalized) return fail(ODY_ERR_STATE, "context not finalized");
  *njobs = (int64_t)c->jobs.size();
  if (grid) *grid = c->grid_apply;
  if (jobs_out) {
    if (cap < (int64_t)c->jobs.size()) return fail(ODY_ERR_ARG, "job buffer too small");
    std::copy(c->jobs.begin(), c->jobs.end(), jobs_out);
  }
  return ODY_OK;
}

static void drop_graph(ody_ctx* c);

// Test hook for the device-side bounded wait: replaces the context's job
// list (NULL: back to the planned list) and the bound on a requant job's
// readiness wait (wait_ns 0: the 2 s default).  Entries are checked against
// the chunk table; a requant entry must name a chunk of a per-tensor-scaled
// tensor.  A list that leaves out some update job of a tensor whose requant
// job it keeps makes that wait run out, which ody_step_wait reports as
// ODY_ERR_DEVICE_BOUNDS.
extern "C" int odyx_ctx_set_jobs(ody_ctx* c, const uint32_t* jobs, int64_t n, uint64_t wait_ns) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (c->pending) return ctx_fail(c, ODY_ERR_STATE, "a step is in flight");
  if (jobs) {
    if (n < 0 || n > (int64_t)INT32_MAX) return ctx_fail(c, ODY_ERR_ARG, "bad job count");
    for (int64_t i = 0; i < n; i++) {
      const uint32_t ch = jobs[i] & ~kRequantJob;
      if (ch >= c->chunks_upd.size()) return ctx_fail(c, ODY_ERR_ARG, "job " + std::to_string(i) + ": bad chunk");
      const int q = c->tdesc[c->chunks_upd[ch].tensor].quant;
      if ((jobs[i] & kRequantJob) && q != Q_FP8_E4M3_TENSOR && q != Q_NVFP4_TENSOR)
        return ctx_fail(c, ODY_ERR_ARG, "job " + std::to_string(i) + ": requant of a tensor without a per-tensor scale");
    }
    c->jobs.assign(jobs, jobs + n);
  } else {
    build_jobs(c);
  }
  c->wait_ns = wait_ns ? (unsigned long long)wait_ns : kWaitLimitNs;
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (c->gexec) {
    ODY_CUDA(cudaStreamSynchronize(c->stream));
    drop_graph(c);
  }
  return upload_jobs(c);
}

extern "C" int ody_ctx_finalize(ody_ctx* c, int32_t world, int32_t rank, const void* uid) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context already finalized");
  if (c->specs.empty()) return ctx_fail(c, ODY_ERR_SHAPE, "no tensors registered");
  if (world < 1 || rank < 0 || rank >= world) return ctx_fail(c, ODY_ERR_ARG, "bad world_size/rank");
  if (world > 1 && !uid) return ctx_fail(c, ODY_ERR_ARG, "nccl_unique_id required when world_size > 1");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  c->world = world;
  c->rank = rank;
  const int nt = (int)c->specs.size();
  c->owner.assign(nt, 0);
  std::vector<int64_t> numels(nt);
  for (int i = 0; i < nt; i++) numels[i] = c->specs[i].numel;
  ody_plan_shards(numels.data(), nt, world, c->owner.data());
  c->local_of.assign(nt, -1);
  // chunk length: 32 tiles, halved while the model would give fewer than four
  // chunks per resident apply CTA (small models spread over more CTAs
  // instead of walking long chunks tile by tile)
  int64_t chunk = kChunk;
  {
    int64_t nloc = 0;
    for (int i = 0; i < nt; i++)
      if (c->owner[i] == rank) nloc += (c->specs[i].numel + kPad - 1) / kPad * kPad;
    const int64_t full = apply_grid(c->gdt, c->cfg.optimizer, c->cfg.device);
    while (chunk > kTile && nloc / chunk < 4 * full) chunk /= 2;
    if (c->cfg.chunk_elems > 0) chunk = c->cfg.chunk_elems;  // validated at create
  }
  int64_t off = 0, qoff = 0;
  for (int i = 0; i < nt; i++) {
    if (c->owner[i] != rank) continue;
    TensorDesc d;
    memset(&d, 0, sizeof(d));
    d.numel = c->specs[i].numel;
    d.npad = (d.numel + kPad - 1) / kPad * kPad;
    d.off = off;
    d.qoff = qoff;
    d.quant = c->specs[i].quant;
    c->local_of[i] = (int32_t)c->tdesc.size();
    const int li = (int)c->tdesc.size();
    c->tdesc.push_back(d);
    for (int64_t s = 0; s < d.npad; s += chunk) {
      Chunk ch;
      ch.start = d.off + s;
      ch.len = (int32_t)((d.npad - s) < chunk ? (d.npad - s) : chunk);
      ch.tensor = li;
      c->chunks_upd.push_back(ch);
      c->tdesc[li].nchunks++;
    }
    off += d.npad;
    qoff += quant_region(d.quant, d.npad);
  }
  c->n_total = off;
  c->q_total = qoff;
  c->gq_off.assign(nt, 0);
  c->rank_qbeg.assign(world, 0);
  c->rank_qend.assign(world, 0);
  c->rank_tbeg.assign(world, 0);
  c->rank_tend.assign(world, 0);
  {
    int64_t g = 0;
    std::vector<bool> seen(world, false);
    for (int i = 0; i < nt; i++) {
      const int r = c->owner[i];
      const int64_t npad = (c->specs[i].numel + kPad - 1) / kPad * kPad;
      if (!seen[r]) {
        seen[r] = true;
        c->rank_qbeg[r] = g;
        c->rank_tbeg[r] = i;
      }
      c->gq_off[i] = g;
      g += quant_region(c->specs[i].quant, npad);
      c->rank_qend[r] = g;
      c->rank_tend[r] = i + 1;
    }
    for (int r = 0; r < world; r++)
      if (!seen[r]) c->rank_qbeg[r] = c->rank_qend[r] = g, c->rank_tbeg[r] = c->rank_tend[r] = nt;
    c->gq_total = g;
  }
  const int nl = (int)c->tdesc.size();
  // a blocking stream: work on it is ordered after work the caller queued on
  // the legacy default stream (e.g. PyTorch producing a device buffer that
  // ody_upload then copies), and vice versa
  ODY_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamDefault));
  ODY_CUDA(cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming));
  const size_t n = (size_t)(off > 0 ? off : kPad);
  const int opt = c->cfg.optimizer;
  const bool need_s1 = opt != ODY_SGD || c->cfg.momentum > 0.0;
  const bool need_s2 = opt == ODY_ADAM || opt == ODY_ADAMW || (opt == ODY_RMSPROP && c->cfg.momentum > 0.0);
  ODY_CUDA(dalloc(&c->master, n * 4));
  ODY_CUDA(cudaMemsetAsync(c->master, 0, n * 4, c->stream));
  if (need_s1) {
    ODY_CUDA(dalloc(&c->s1, n * 4));
    ODY_CUDA(cudaMemsetAsync(c->s1, 0, n * 4, c->stream));
  }
  if (need_s2) {
    ODY_CUDA(dalloc(&c->s2, n * 4));
    ODY_CUDA(cudaMemsetAsync(c->s2, 0, n * 4, c->stream));
  }
  ODY_CUDA(dalloc(&c->grad, n * dtype_size(c->gdt)));
  ODY_CUDA(cudaMemsetAsync(c->grad, 0, n * dtype_size(c->gdt), c->stream));
  ODY_CUDA(dalloc(&c->qout, (size_t)qoff));
  ODY_CUDA(cudaMemsetAsync(c->qout, 0, (size_t)(qoff > 0 ? qoff : 256), c->stream));
  ODY_CUDA(dalloc(&c->qscale, sizeof(float) * (nl > 0 ? nl : 1)));
  std::vector<float> ones(nl > 0 ? nl : 1, 1.0f);
  ODY_CUDA(cudaMemcpyAsync(c->qscale, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice, c->stream));
  ODY_CUDA(dalloc(&c->amax, sizeof(uint32_t) * (nl > 0 ? nl : 1)));
  ODY_CUDA(cudaMemsetAsync(c->amax, 0, sizeof(uint32_t) * (nl > 0 ? nl : 1), c->stream));
  ODY_CUDA(dalloc(&c->d_tdesc, sizeof(TensorDesc) * (nl > 0 ? nl : 1)));
  if (nl) ODY_CUDA(cudaMemcpyAsync(c->d_tdesc, c->tdesc.data(), sizeof(TensorDesc) * nl, cudaMemcpyHostToDevice, c->stream));
  ODY_CUDA(dalloc(&c->d_chunks_upd, sizeof(Chunk) * (c->chunks_upd.size() + 1)));
  if (!c->chunks_upd.empty())
    ODY_CUDA(cudaMemcpyAsync(c->d_chunks_upd, c->chunks_upd.data(), sizeof(Chunk) * c->chunks_upd.size(),
                             cudaMemcpyHostToDevice, c->stream));
  // a model smaller than one chunk per resident CTA launches one CTA per
  // update chunk: idle CTAs of a persistent grid only add launch latency
  c->grid_apply = apply_grid(c->gdt, c->cfg.optimizer, c->cfg.device);
  if ((size_t)c->grid_apply > c->chunks_upd.size()) c->grid_apply = (int)std::max<size_t>(1, c->chunks_upd.size());
  build_jobs(c);
  {
    const int rc = upload_jobs(c);
    if (rc) return rc;
  }
  ODY_CUDA(dalloc(&c->sync, sizeof(uint32_t) * (nl + 1)));
  ODY_CUDA(cudaMemsetAsync(c->sync, 0, sizeof(uint32_t) * (nl + 1), c->stream));
  // one unrolled round (4 groups of 8 gradients) per thread, at most the
  // resident grid (the fixed-order partial reduction makes the sum depend on
  // the grid, which is fixed for the context's lifetime)
  {
    const int64_t per_cta = (int64_t)kThreads * 4 * 8;
    const int64_t want = (c->n_total + per_cta - 1) / per_cta;
    c->grid_stats = (int)std::max<int64_t>(1, std::min<int64_t>(stats_grid(c->cfg.device), want));
  }
  ODY_CUDA(dalloc(&c->partials, sizeof(StatsPartial) * c->grid_stats));
  ODY_CUDA(dalloc(&c->ticket, sizeof(unsigned)));
  ODY_CUDA(cudaMemsetAsync(c->ticket, 0, sizeof(unsigned), c->stream));
  ODY_CUDA(dalloc(&c->scaler, sizeof(DevScaler)));
  DevScaler hs;
  memset(&hs, 0, sizeof(hs));
  hs.scale = c->cfg.initial_scale;
  ODY_CUDA(cudaMemcpyAsync(c->scaler, &hs, sizeof(hs), cudaMemcpyHostToDevice, c->stream));
  ODY_CUDA(dalloc(&c->dec, sizeof(Decision)));
  ODY_CUDA(cudaMemsetAsync(c->dec, 0, sizeof(Decision), c->stream));
  ODY_CUDA(dalloc(&c->local_stats, sizeof(double) * 2));
  ODY_CUDA(dalloc(&c->gathered, sizeof(double) * 2 * world));
  ODY_CUDA(cudaMallocHost((void**)&c->h_dec, sizeof(Decision)));
  upload_fp4_tables(c->cfg.device);
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  if (world > 1) {
    std::string why;
    NcclApi* api = nccl_api(why);
    if (!api) return ctx_fail(c, ODY_ERR_NCCL, why);
    ncclUniqueId id;
    memcpy(&id, uid, sizeof(id));
    ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
    conf.blocking = 0;
    ncclResult_t r = api->commInitRankConfig(&c->comm, world, id, rank, &conf);
    if (r != ncclSuccess && r != ncclInProgress)
      return ctx_fail(c, ODY_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + api->getErrorString(r));
    int rc = wait_nccl(c, api, "ncclCommInitRankConfig");
    if (rc != ODY_OK) return rc;
  }
  c->finalized = true;
  return ODY_OK;
}

extern "C" int ody_ctx_tensor_owner(const ody_ctx* c, int32_t i, int32_t* r) {
  if (!c || !r) return fail(ODY_ERR_ARG, "null argument");
  if (!c->finalized) return fail(ODY_ERR_STATE, "context not finalized");
  if (i < 0 || i >= (int)c->specs.size()) return fail(ODY_ERR_ARG, "tensor index out of range");
  *r = c->owner[i];
  return ODY_OK;
}

extern "C" int ody_ctx_num_tensors(const ody_ctx* c, int32_t* n) {
  if (!c || !n) return fail(ODY_ERR_ARG, "null argument");
  *n = (int32_t)c->specs.size();
  return ODY_OK;
}

static int locate(ody_ctx* c, int32_t which, int32_t i, void** base, size_t* bytes) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (i < 0 || i >= (int)c->specs.size()) return ctx_fail(c, ODY_ERR_ARG, "tensor index out of range");
  if (which == ODY_BUF_DP_GRAD) {
    if (!c->dp_on) return ctx_fail(c, ODY_ERR_STATE, "data-parallel gradients not attached (ody_ctx_dp_attach)");
    *base = (uint8_t*)c->dp_buf + (size_t)c->dp_off[i] * dtype_size(c->gdt);
    *bytes = (size_t)c->specs[i].numel * dtype_size(c->gdt);
    return ODY_OK;
  }
  const int li = c->local_of[i];
  if (li < 0)
    return ctx_fail(c, ODY_ERR_ARG, "tensor " + std::to_string(i) + " is owned by rank " +
                                        std::to_string(c->owner[i]));
  const TensorDesc& d = c->tdesc[li];
  switch (which) {
    case ODY_BUF_MASTER:
      *base = c->master + d.off;
      *bytes = (size_t)d.numel * 4;
      break;
    case ODY_BUF_STATE1:
      if (!c->s1) return ctx_fail(c, ODY_ERR_ARG, "optimizer has no first state buffer");
      *base = c->s1 + d.off;
      *bytes = (size_t)d.numel * 4;
      break;
    case ODY_BUF_STATE2:
      if (!c->s2) return ctx_fail(c, ODY_ERR_ARG, "optimizer has no second state buffer");
      *base = c->s2 + d.off;
      *bytes = (size_t)d.numel * 4;
      break;
    case ODY_BUF_GRAD:
      *base = (uint8_t*)step_grad(c) + (size_t)d.off * dtype_size(c->gdt);
      *bytes = (size_t)d.numel * dtype_size(c->gdt);
      break;
    default:
      return ctx_fail(c, ODY_ERR_ARG, "unknown buffer " + std::to_string(which));
  }
  return ODY_OK;
}

static int copy_tensor(ody_ctx* c, int32_t which, int32_t i, void* dst_or_src, size_t bytes, bool up,
                       bool sync) {
  void* base;
  size_t need;
  int rc = locate(c, which, i, &base, &need);
  if (rc) return rc;
  if (bytes != need)
    return ctx_fail(c, ODY_ERR_SHAPE, "size mismatch: expected " + std::to_string(need) + " bytes, got " +
                                          std::to_string(bytes));
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (c->dbuf && which == ODY_BUF_GRAD) {
    // the copy stream: after the step that last read this arena, and ahead
    // of the step that reads it next (which waits on slot_filled)
    const int s = c->upload_slot;
    if (!c->slot_ordered) {  // once per step, not once per tensor
      ODY_CUDA(cudaStreamWaitEvent(c->copy_stream, c->slot_read[s], 0));
      c->slot_ordered = true;
    }
    if (up)
      ODY_CUDA(cudaMemcpyAsync(base, dst_or_src, bytes, cudaMemcpyDefault, c->copy_stream));
    else
      ODY_CUDA(cudaMemcpyAsync(dst_or_src, base, bytes, cudaMemcpyDefault, c->copy_stream));
    if (sync) ODY_CUDA(cudaStreamSynchronize(c->copy_stream));
    return ODY_OK;
  }
  if (up)
    ODY_CUDA(cudaMemcpyAsync(base, dst_or_src, bytes, cudaMemcpyDefault, c->stream));
  else
    ODY_CUDA(cudaMemcpyAsync(dst_or_src, base, bytes, cudaMemcpyDefault, c->stream));
  if (sync) ODY_CUDA(cudaStreamSynchronize(c->stream));
  return ODY_OK;
}

extern "C" int ody_upload(ody_ctx* c, int32_t which, int32_t i, const void* src, size_t bytes) {
  return copy_tensor(c, which, i, const_cast<void*>(src), bytes, true, true);
}
extern "C" int ody_upload_async(ody_ctx* c, int32_t which, int32_t i, const void* src, size_t bytes) {
  return copy_tensor(c, which, i, const_cast<void*>(src), bytes, true, false);
}
extern "C" int ody_download(ody_ctx* c, int32_t which, int32_t i, void* dst, size_t bytes) {
  return copy_tensor(c, which, i, dst, bytes, false, true);
}

extern "C" int ody_ctx_device_ptr(ody_ctx* c, int32_t which, int32_t i, void** out) {
  if (!out) return fail(ODY_ERR_ARG, "null output");
  size_t b;
  return locate(c, which, i, out, &b);
}

extern "C" int ody_ctx_stream(ody_ctx* c, void** out) {
  if (!c || !out) return fail(ODY_ERR_ARG, "null argument");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  *out = (void*)c->stream;
  return ODY_OK;
}

// Optimizer constants: Float64 hyper-parameters rounded once to float32
// (full_like, tensor_creation.mojo:355-376); bias corrections
// 1 - beta^t computed in Float64 (adam.mojo:142-152).
static OptConsts make_consts(const ody_config& cfg, int64_t t) {
  OptConsts o;
  memset(&o, 0, sizeof(o));
  o.lr = (float)cfg.learning_rate;
  o.mu = (float)cfg.momentum;
  o.wd = (float)cfg.weight_decay;
  o.use_wd = cfg.weight_decay > 0.0;
  o.use_mu = cfg.momentum > 0.0;
  o.b1 = (float)cfg.beta1;
  o.omb1 = (float)(1.0 - cfg.beta1);
  o.b2 = (float)cfg.beta2;
  o.omb2 = (float)(1.0 - cfg.beta2);
  o.eps = (float)cfg.epsilon;
  o.alpha = (float)cfg.alpha;
  o.omalpha = (float)(1.0 - cfg.alpha);
  o.wdlr = (float)(cfg.weight_decay * cfg.learning_rate);
  o.use_wd_nz = cfg.weight_decay != 0.0;
  if (t > 0 && (cfg.optimizer == ODY_ADAM || cfg.optimizer == ODY_ADAMW)) {
    o.bc1 = (float)(1.0 - pow(cfg.beta1, (double)t));
    o.bc2 = (float)(1.0 - pow(cfg.beta2, (double)t));
  }
  return o;
}

static DecideParams make_decide(const ody_config& cfg) {
  DecideParams d;
  memset(&d, 0, sizeof(d));
  d.use_scaler = cfg.use_gradient_scaler;
  d.clip_enabled = cfg.clip_enabled;
  d.max_norm = cfg.max_norm;
  d.growth_factor = cfg.growth_factor;
  d.backoff_factor = cfg.backoff_factor;
  d.min_scale = cfg.min_scale;
  d.max_scale = cfg.max_scale;
  d.growth_interval = cfg.growth_interval;
  return d;
}

// pass 1: the stats kernel over the local gradients, or with data-parallel
// gradients attached the fused reduce-scatter + stats kernel
static cudaError_t launch_pass1(ody_ctx* c, const DecideParams& dp, int world_mode) {
  const int nl = (int)c->tdesc.size();
  if (c->dp_on)
    return launch_rs_stats(c->gdt, c->d_peers, c->world, c->dp_shard_off, step_grad(c), c->n_total,
                           c->cfg.use_gradient_scaler, c->scaler, c->partials, c->grid_stats, c->ticket, world_mode,
                           c->local_stats, dp, c->dec, c->amax, c->sync, nl, c->stream);
  return launch_stats(c->gdt, step_grad(c), c->n_total, c->cfg.use_gradient_scaler, c->scaler, c->partials,
                      c->grid_stats, c->ticket, world_mode, c->local_stats, dp, c->dec, c->amax, c->sync, nl,
                      c->stream);
}

static void drop_graph(ody_ctx* c) {
  if (c->gexec) cudaGraphExecDestroy(c->gexec);
  if (c->graph) cudaGraphDestroy(c->graph);
  c->gexec = nullptr;
  c->graph = nullptr;
  c->gapply = nullptr;
}

// One step as one graph launch (one GPU).  The first call captures stats ->
// apply -> result read-back from the context's stream; later calls update the
// apply node's arguments when the optimizer constants of step t differ and
// relaunch.
static int step_graph(ody_ctx* c, const OptConsts& oc, const DecideParams& dp) {
  const int nl = (int)c->tdesc.size();
  if (!c->gexec) {
    ODY_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = launch_pass1(c, dp, 0);
    if (e == cudaSuccess)
      e = launch_apply(c->gdt, c->cfg.optimizer, oc, c->cfg.use_gradient_scaler, c->d_chunks_upd, c->d_jobs,
                       (int)c->jobs.size(), c->d_tdesc, c->master, c->s1, c->s2, c->grad, c->qout, c->amax,
                       c->qscale, c->sync, c->dec, c->grid_apply, c->stream, c->wait_ns);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(c->h_dec, c->dec, sizeof(Decision), cudaMemcpyDeviceToHost, c->stream);
    cudaGraph_t g = nullptr;
    const cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return ctx_fail(c, ODY_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    }
    c->graph = g;
    size_t n = 0;
    ODY_CUDA(cudaGraphGetNodes(g, nullptr, &n));
    std::vector<cudaGraphNode_t> nodes(n);
    ODY_CUDA(cudaGraphGetNodes(g, nodes.data(), &n));
    const void* fn = apply_kernel_fn(c->gdt, c->cfg.optimizer);
    for (cudaGraphNode_t nd : nodes) {
      cudaGraphNodeType ty;
      ODY_CUDA(cudaGraphNodeGetType(nd, &ty));
      if (ty != cudaGraphNodeTypeKernel) continue;
      cudaKernelNodeParams kp;
      ODY_CUDA(cudaGraphKernelNodeGetParams(nd, &kp));
      if (kp.func == fn) c->gapply = nd;
    }
    if (!c->gapply) {
      drop_graph(c);
      return ctx_fail(c, ODY_ERR_CUDA, "graph capture: apply kernel node not found");
    }
    e = cudaGraphInstantiate(&c->gexec, g, 0);
    if (e != cudaSuccess) {
      c->gexec = nullptr;
      drop_graph(c);
      return ctx_fail(c, ODY_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    }
    c->goc = oc;
  } else if (memcmp(&c->goc, &oc, sizeof(OptConsts)) != 0) {
    ODY_CUDA(set_apply_node(c->gexec, c->gapply, c->gdt, c->cfg.optimizer, oc, c->cfg.use_gradient_scaler,
                            c->d_chunks_upd, c->d_jobs, (int)c->jobs.size(), c->d_tdesc, c->master, c->s1, c->s2,
                            c->grad, c->qout, c->amax, c->qscale, c->sync, c->dec, c->grid_apply, c->wait_ns));
    c->goc = oc;
  }
  ODY_CUDA(cudaGraphLaunch(c->gexec, c->stream));
  ODY_CUDA(cudaEventRecord(c->done, c->stream));
  c->pending = true;
  return ODY_OK;
}

// the data-parallel buffers and peer mappings (also after a failed attach)
static void dp_release(ody_ctx* c) {
  for (void* p : c->dp_opened) cudaIpcCloseMemHandle(p);
  c->dp_opened.clear();
  void* dpb[] = {c->dp_buf, (void*)c->d_peers, c->bar_send, c->bar_recv};
  for (void* b : dpb)
    if (b) cudaFree(b);
  c->dp_buf = nullptr;
  c->d_peers = nullptr;
  c->bar_send = c->bar_recv = nullptr;
  c->dp_on = false;
}

extern "C" int ody_ctx_dp_attach(ody_ctx* c) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (c->broken) return ctx_fail(c, ODY_ERR_STATE, "context unusable after a communicator failure");
  if (c->dp_on) return ctx_fail(c, ODY_ERR_STATE, "data-parallel gradients already attached");
  if (c->dbuf) return ctx_fail(c, ODY_ERR_STATE, "data-parallel gradients do not combine with double-buffered gradients");
  if (c->world > 8) return ctx_fail(c, ODY_ERR_ARG, "data-parallel gradients support at most 8 ranks");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  dp_release(c);  // what a failed earlier attempt left
  const int nt = (int)c->specs.size();
  const size_t esz = dtype_size(c->gdt);
  c->dp_off.assign(nt, 0);
  int64_t g = 0;
  for (int i = 0; i < nt; i++) {
    c->dp_off[i] = g;
    g += (c->specs[i].numel + kPad - 1) / kPad * kPad;
  }
  c->dp_total = g;
  const int r = c->rank;
  c->dp_shard_off = c->rank_tend[r] > c->rank_tbeg[r] ? c->dp_off[c->rank_tbeg[r]] : 0;
  for (int i = 0; i < nt; i++)
    if (c->local_of[i] >= 0 && c->dp_off[i] - c->dp_shard_off != c->tdesc[c->local_of[i]].off)
      return ctx_fail(c, ODY_ERR_STATE, "shard is not contiguous in the global layout");
  ODY_CUDA(dalloc(&c->dp_buf, (size_t)g * esz));
  ODY_CUDA(cudaMemsetAsync(c->dp_buf, 0, (size_t)g * esz, c->stream));
  std::vector<const void*> peers(c->world, nullptr);
  peers[r] = c->dp_buf;
  if (c->world > 1) {
    std::string why;
    NcclApi* api = nccl_api(why);
    if (!api) return ctx_fail(c, ODY_ERR_NCCL, why);
    cudaIpcMemHandle_t h;
    ODY_CUDA(cudaIpcGetMemHandle(&h, c->dp_buf));
    uint8_t* dh = nullptr;
    ODY_CUDA(dalloc(&dh, sizeof(h) * (c->world + 1)));
    ODY_CUDA(cudaMemcpyAsync(dh, &h, sizeof(h), cudaMemcpyHostToDevice, c->stream));
    ncclResult_t nr = api->allGather(dh, dh + sizeof(h), sizeof(h), ncclUint8, c->comm, c->stream);
    if (nr != ncclSuccess && nr != ncclInProgress) {
      cudaFree(dh);
      return ctx_fail(c, ODY_ERR_NCCL, std::string("ncclAllGather (IPC handles): ") + api->getErrorString(nr));
    }
    int rc = wait_nccl(c, api, "ncclAllGather (IPC handles)");
    if (rc != ODY_OK) {
      cudaFree(dh);
      return rc;
    }
    std::vector<cudaIpcMemHandle_t> all(c->world);
    cudaError_t e = cudaMemcpyAsync(all.data(), dh + sizeof(h), sizeof(h) * c->world, cudaMemcpyDeviceToHost,
                                    c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(dh);
    if (e != cudaSuccess) return ctx_fail(c, ODY_ERR_CUDA, std::string("IPC handles: ") + cudaGetErrorString(e));
    for (int q = 0; q < c->world; q++) {
      if (q == r) continue;
      void* p = nullptr;
      e = cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess)
        return ctx_fail(c, ODY_ERR_CUDA, "opening rank " + std::to_string(q) +
                                             "'s gradient buffer (peer access over NVLink required): " +
                                             cudaGetErrorString(e));
      c->dp_opened.push_back(p);
      peers[q] = p;
    }
    ODY_CUDA(dalloc(&c->bar_send, sizeof(double)));
    ODY_CUDA(dalloc(&c->bar_recv, sizeof(double) * c->world));
    ODY_CUDA(cudaMemsetAsync(c->bar_send, 0, sizeof(double), c->stream));
  }
  ODY_CUDA(dalloc(&c->d_peers, sizeof(void*) * c->world));
  ODY_CUDA(cudaMemcpyAsync(c->d_peers, peers.data(), sizeof(void*) * c->world, cudaMemcpyHostToDevice, c->stream));
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  if (c->gexec) drop_graph(c);  // the captured pass 1 changes
  c->dp_on = true;
  return ODY_OK;
}

extern "C" int ody_ctx_set_grad_double_buffer(ody_ctx* c, int32_t enable) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (c->pending) return ctx_fail(c, ODY_ERR_STATE, "a step is in flight");
  if (c->dp_on) return ctx_fail(c, ODY_ERR_STATE, "double-buffered gradients do not combine with data-parallel gradients");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (c->gexec && enable != (int32_t)c->dbuf) {
    // a captured step names the old gradient arena: capture again later
    ODY_CUDA(cudaStreamSynchronize(c->stream));
    drop_graph(c);
  }
  if (!enable) {
    if (!c->dbuf) return ODY_OK;
    ODY_CUDA(cudaStreamSynchronize(c->copy_stream));
    ODY_CUDA(cudaStreamSynchronize(c->stream));
    // the arena the next step would read becomes the single arena
    if (c->upload_slot == 1) std::swap(c->grad_slot[0], c->grad_slot[1]);
    c->grad = c->grad_slot[0];
    ODY_CUDA(cudaFree(c->grad_slot[1]));
    c->grad_slot[1] = nullptr;
    c->upload_slot = 0;
    c->slot_ordered = false;
    c->dbuf = false;
    return ODY_OK;
  }
  if (c->dbuf) return ODY_OK;
  const size_t bytes = (size_t)(c->n_total > 0 ? c->n_total : kPad) * dtype_size(c->gdt);
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  if (!c->copy_stream) {
    ODY_CUDA(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
    for (int s = 0; s < 2; s++) {
      ODY_CUDA(cudaEventCreateWithFlags(&c->slot_read[s], cudaEventDisableTiming));
      ODY_CUDA(cudaEventCreateWithFlags(&c->slot_filled[s], cudaEventDisableTiming));
      ODY_CUDA(cudaEventRecord(c->slot_read[s], c->stream));
      ODY_CUDA(cudaEventRecord(c->slot_filled[s], c->stream));
    }
  }
  void* alt = nullptr;
  ODY_CUDA(dalloc((uint8_t**)&alt, bytes));
  ODY_CUDA(cudaMemsetAsync(alt, 0, bytes, c->stream));
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  c->grad_slot[0] = c->grad;
  c->grad_slot[1] = alt;
  c->upload_slot = 0;
  c->slot_ordered = false;
  c->dbuf = true;
  return ODY_OK;
}

extern "C" int ody_ctx_set_graph(ody_ctx* c, int32_t enable) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (!enable && c->gexec) {
    ODY_CUDA(cudaStreamSynchronize(c->stream));
    drop_graph(c);
  }
  c->graph_mode = enable != 0;
  return ODY_OK;
}

extern "C" int ody_step_async(ody_ctx* c, int64_t t) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (c->broken) return ctx_fail(c, ODY_ERR_STATE, "context unusable after a communicator failure");
  if (needs_timestep(c->cfg.optimizer) && t <= 0)
    return ctx_fail(c, ODY_ERR_ARG, "Timestep t must be positive (starts at 1)");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  const OptConsts oc = make_consts(c->cfg, t);
  const DecideParams dp = make_decide(c->cfg);
  const int nl = (int)c->tdesc.size();
  if (c->graph_mode && c->world == 1 && !c->timing && !c->dbuf && !c->jobs.empty()) return step_graph(c, oc, dp);
  if (c->dbuf) {
    // the step reads the slot after every upload queued into it so far
    ODY_CUDA(cudaEventRecord(c->slot_filled[c->upload_slot], c->copy_stream));
    ODY_CUDA(cudaStreamWaitEvent(c->stream, c->slot_filled[c->upload_slot], 0));
  }
  cudaEvent_t* tev = nullptr;
  if (c->timing) {
    const int64_t slot = c->tnext++;
    if (!c->tpending.empty() && c->tpending.front() + kTimingRing <= slot) {
      ODY_CUDA(timing_collect(c, c->tpending.front()));
      c->tpending.erase(c->tpending.begin());
    }
    c->tpending.push_back(slot);
    tev = &c->tev[(size_t)(slot % kTimingRing) * 5];
    ODY_CUDA(cudaEventRecord(tev[0], c->stream));
  }
  cudaError_t e;
  if (c->dp_on && c->world > 1) {
    // every rank's gradients are written before any rank reads them: an
    // 8-byte allgather orders this rank's kernel after every rank's
    // preceding work on its stream
    std::string why;
    NcclApi* api = nccl_api(why);
    if (!api) return ctx_fail(c, ODY_ERR_NCCL, why);
    ncclResult_t r = api->allGather(c->bar_send, c->bar_recv, 1, ncclFloat64, c->comm, c->stream);
    if (r != ncclSuccess && r != ncclInProgress)
      return ctx_fail(c, ODY_ERR_NCCL, std::string("ncclAllGather (gradient barrier): ") + api->getErrorString(r));
    int rc = wait_nccl(c, api, "ncclAllGather (gradient barrier)");
    if (rc != ODY_OK) return rc;
  }
  e = launch_pass1(c, dp, c->world > 1 ? 1 : 0);
  if (e != cudaSuccess) return ctx_fail(c, ODY_ERR_CUDA, std::string("stats kernel: ") + cudaGetErrorString(e));
  if (tev) ODY_CUDA(cudaEventRecord(tev[1], c->stream));
  if (c->world > 1) {
    std::string why;
    NcclApi* api = nccl_api(why);
    if (!api) return ctx_fail(c, ODY_ERR_NCCL, why);
    ncclResult_t r = api->allGather(c->local_stats, c->gathered, 2, ncclFloat64, c->comm, c->stream);
    if (r != ncclSuccess && r != ncclInProgress)
      return ctx_fail(c, ODY_ERR_NCCL, std::string("ncclAllGather: ") + api->getErrorString(r));
    int rc = wait_nccl(c, api, "ncclAllGather");
    if (rc != ODY_OK) return rc;
    e = launch_finalize(c->gathered, c->world, c->scaler, dp, c->dec, c->amax, nl, c->stream);
    if (e != cudaSuccess) return ctx_fail(c, ODY_ERR_CUDA, std::string("finalize kernel: ") + cudaGetErrorString(e));
  }
  if (tev) ODY_CUDA(cudaEventRecord(tev[2], c->stream));
  if (!c->jobs.empty()) {
    e = launch_apply(c->gdt, c->cfg.optimizer, oc, c->cfg.use_gradient_scaler, c->d_chunks_upd, c->d_jobs,
                     (int)c->jobs.size(), c->d_tdesc, c->master, c->s1, c->s2, step_grad(c), c->qout, c->amax, c->qscale,
                     c->sync, c->dec, c->grid_apply, c->stream, c->wait_ns);
    if (e != cudaSuccess) return ctx_fail(c, ODY_ERR_CUDA, std::string("apply kernel: ") + cudaGetErrorString(e));
  }
  if (tev) ODY_CUDA(cudaEventRecord(tev[3], c->stream));
  if (tev) ODY_CUDA(cudaEventRecord(tev[4], c->stream));
  if (c->dbuf) {
    // this step's arena is free for uploads once the apply kernel is done;
    // the next step reads the other one
    ODY_CUDA(cudaEventRecord(c->slot_read[c->upload_slot], c->stream));
    c->upload_slot ^= 1;
    c->slot_ordered = false;
  }
  ODY_CUDA(cudaMemcpyAsync(c->h_dec, c->dec, sizeof(Decision), cudaMemcpyDeviceToHost, c->stream));
  ODY_CUDA(cudaEventRecord(c->done, c->stream));
  c->pending = true;
  return ODY_OK;
}

static void fill_result(const Decision& d, ody_step_result* o) {
  memset(o, 0, sizeof(*o));
  o->found_inf = d.nonfinite > 0;
  o->skipped = d.skip;
  o->clipped = d.clipped;
  o->nonfinite_count = d.nonfinite;
  o->sumsq = d.sumsq;
  o->grad_norm = d.norm;
  o->clip_coef = d.coef;
  o->scale_used = d.scale_used;
  o->scale_next = d.scale_next;
  o->step_count = d.step_count;
  o->overflow_count = d.overflow_count;
  o->scaler_num_steps = d.scaler_num_steps;
  o->steps_since_growth = d.steps_since_growth;
}

extern "C" int ody_step_wait(ody_ctx* c, ody_step_result* out) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->pending) return ctx_fail(c, ODY_ERR_STATE, "no step in flight");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (c->world > 1) {
    // bounded host-side wait: a peer that stopped answering aborts the
    // communicator instead of hanging this rank
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      cudaError_t q = cudaEventQuery(c->done);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return ctx_fail(c, ODY_ERR_CUDA, std::string("step: ") + cudaGetErrorString(q));
      std::string why;
      NcclApi* api = nccl_api(why);
      ncclResult_t st = ncclSuccess;
      if (api && c->comm) api->commGetAsyncError(c->comm, &st);
      auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if ((st != ncclSuccess && st != ncclInProgress) || ms > c->cfg.comm_timeout_ms) {
        const bool failed = st != ncclSuccess && st != ncclInProgress;
        const std::string what = failed ? std::string("step: communicator failed: ") + api->getErrorString(st)
                                        : "step: no completion within " + std::to_string(c->cfg.comm_timeout_ms) +
                                              " ms";
        if (api && c->comm) api->commAbort(c->comm);
        c->comm = nullptr;
        c->broken = true;
        c->pending = false;
        return ctx_fail(c, failed ? ODY_ERR_NCCL : ODY_ERR_COMM_TIMEOUT, what);
      }
    }
  } else {
    ODY_CUDA(cudaEventSynchronize(c->done));
  }
  c->pending = false;
  if (out) fill_result(*c->h_dec, out);
  if (c->h_dec->err)
    return ctx_fail(c, ODY_ERR_DEVICE_BOUNDS,
                    "apply kernel: a requant job waited past its time limit for its tensor's update");
  return ODY_OK;
}

extern "C" int ody_step(ody_ctx* c, int64_t t, ody_step_result* out) {
  int rc = ody_step_async(c, t);
  if (rc) return rc;
  return ody_step_wait(c, out);
}

extern "C" int ody_ctx_set_timing(ody_ctx* c, int32_t enable) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (enable && c->tev.empty()) {
    c->tev.resize((size_t)kTimingRing * 5);
    for (auto& e : c->tev) ODY_CUDA(cudaEventCreate(&e));
  }
  c->timing = enable != 0;
  return ODY_OK;
}

extern "C" int ody_ctx_pass_times(ody_ctx* c, double* ms_out, int64_t* steps_out) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  for (int64_t slot : c->tpending) ODY_CUDA(timing_collect(c, slot));
  c->tpending.clear();
  if (ms_out)
    for (int k = 0; k < 4; k++) ms_out[k] = c->tms[k];
  if (steps_out) *steps_out = c->tsteps;
  for (int k = 0; k < 4; k++) c->tms[k] = 0.0;
  c->tsteps = 0;
  return ODY_OK;
}

extern "C" int ody_ctx_quant_layout(const ody_ctx* c, int32_t i, int64_t* offset, int64_t* bytes,
                                    int64_t* total) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return fail(ODY_ERR_STATE, "context not finalized");
  if (total) *total = c->gq_total;
  if (i < 0) return ODY_OK;
  if (i >= (int)c->specs.size()) return fail(ODY_ERR_ARG, "tensor index out of range");
  if (offset) *offset = c->gq_off[i];
  if (bytes) *bytes = ody_quant_bytes(c->specs[i].quant, c->specs[i].numel);
  return ODY_OK;
}

extern "C" int ody_ctx_gather_quant(ody_ctx* c, void* dst, float* scales) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (c->broken) return ctx_fail(c, ODY_ERR_STATE, "context unusable after a communicator failure");
  if (!dst || !scales) return ctx_fail(c, ODY_ERR_ARG, "null destination");
  if (!is_device_ptr(dst) || !is_device_ptr(scales))
    return ctx_fail(c, ODY_ERR_ARG, "gather destinations must be device memory of the context's GPU");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  const int r = c->rank;
  const int64_t nb = c->rank_qend[r] - c->rank_qbeg[r];
  const int nts = c->rank_tend[r] - c->rank_tbeg[r];
  if (c->world == 1) {
    if (nb) ODY_CUDA(cudaMemcpyAsync(dst, c->qout, (size_t)nb, cudaMemcpyDeviceToDevice, c->stream));
    if (nts) ODY_CUDA(cudaMemcpyAsync(scales, c->qscale, sizeof(float) * nts, cudaMemcpyDeviceToDevice, c->stream));
    ODY_CUDA(cudaStreamSynchronize(c->stream));
    return ODY_OK;
  }
  std::string why;
  NcclApi* api = nccl_api(why);
  if (!api) return ctx_fail(c, ODY_ERR_NCCL, why);
  // equal slices laid out in rank order (the 1B model on 2/4/8 ranks): one
  // allgather; otherwise one broadcast per rank of its contiguous slice,
  // grouped (an allgather of unequal slices)
  bool eq_codes = true, eq_scales = true;
  for (int q = 0; q < c->world; q++) {
    eq_codes = eq_codes && c->rank_qend[q] - c->rank_qbeg[q] == nb && c->rank_qbeg[q] == (int64_t)q * nb;
    eq_scales = eq_scales && c->rank_tend[q] - c->rank_tbeg[q] == nts && c->rank_tbeg[q] == q * nts;
  }
  api->groupStart();
  if (eq_codes && nb > 0) api->allGather(c->qout, dst, (size_t)nb, ncclUint8, c->comm, c->stream);
  if (eq_scales && nts > 0) api->allGather(c->qscale, scales, (size_t)nts, ncclFloat32, c->comm, c->stream);
  for (int q = 0; q < c->world; q++) {
    const int64_t qb = c->rank_qend[q] - c->rank_qbeg[q];
    if (!eq_codes && qb > 0)
      api->broadcast(q == r ? (const void*)c->qout : nullptr, (uint8_t*)dst + c->rank_qbeg[q], (size_t)qb,
                     ncclUint8, q, c->comm, c->stream);
    const int tq = c->rank_tend[q] - c->rank_tbeg[q];
    if (!eq_scales && tq > 0)
      api->broadcast(q == r ? (const void*)c->qscale : nullptr, scales + c->rank_tbeg[q], (size_t)tq,
                     ncclFloat32, q, c->comm, c->stream);
  }
  ncclResult_t ge = api->groupEnd();
  if (ge != ncclSuccess && ge != ncclInProgress)
    return ctx_fail(c, ODY_ERR_NCCL, std::string("ncclGroupEnd: ") + api->getErrorString(ge));
  int rc = wait_nccl(c, api, "gather of the quantised weights");
  if (rc != ODY_OK) return rc;
  ODY_CUDA(cudaEventRecord(c->done, c->stream));
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaEventQuery(c->done);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return ctx_fail(c, ODY_ERR_CUDA, std::string("gather: ") + cudaGetErrorString(q));
    ncclResult_t st = ncclSuccess;
    api->commGetAsyncError(c->comm, &st);
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if ((st != ncclSuccess && st != ncclInProgress) || ms > c->cfg.comm_timeout_ms) {
      api->commAbort(c->comm);
      c->comm = nullptr;
      c->broken = true;
      return ctx_fail(c, ODY_ERR_COMM_TIMEOUT, "gather of the quantised weights: communicator failed or timed out");
    }
  }
  return ODY_OK;
}

extern "C" int ody_get_quant(ody_ctx* c, int32_t i, void* dst, size_t bytes, float* ts) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  if (i < 0 || i >= (int)c->specs.size()) return ctx_fail(c, ODY_ERR_ARG, "tensor index out of range");
  const int li = c->local_of[i];
  if (li < 0) return ctx_fail(c, ODY_ERR_ARG, "tensor not owned by this rank");
  const TensorDesc& d = c->tdesc[li];
  const int64_t need = ody_quant_bytes(d.quant, d.numel);
  if (d.quant == ODY_Q_NONE) return ctx_fail(c, ODY_ERR_ARG, "tensor has no quantised form");
  if ((int64_t)bytes != need)
    return ctx_fail(c, ODY_ERR_SHAPE, "size mismatch: expected " + std::to_string(need) + " bytes");
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  if (dst) ODY_CUDA(cudaMemcpyAsync(dst, c->qout + d.qoff, bytes, cudaMemcpyDefault, c->stream));
  float s = 1.0f;
  ODY_CUDA(cudaMemcpyAsync(&s, c->qscale + li, 4, cudaMemcpyDeviceToHost, c->stream));
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  if (ts) *ts = s;
  return ODY_OK;
}

extern "C" int ody_get_scaler(ody_ctx* c, float* scale, int64_t* since, int64_t* num, int64_t* steps,
                              int64_t* overflows) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  DevScaler h;
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  ODY_CUDA(cudaMemcpyAsync(&h, c->scaler, sizeof(h), cudaMemcpyDeviceToHost, c->stream));
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  if (scale) *scale = h.scale;
  if (since) *since = h.steps_since_growth;
  if (num) *num = h.num_steps;
  if (steps) *steps = h.step_count;
  if (overflows) *overflows = h.overflow_count;
  return ODY_OK;
}

extern "C" int ody_set_scaler(ody_ctx* c, float scale, int64_t since, int64_t num, int64_t steps,
                              int64_t overflows) {
  if (!c) return fail(ODY_ERR_ARG, "null context");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  DevScaler h;
  memset(&h, 0, sizeof(h));
  h.scale = scale;
  h.steps_since_growth = since;
  h.num_steps = num;
  h.step_count = steps;
  h.overflow_count = overflows;
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  ODY_CUDA(cudaMemcpyAsync(c->scaler, &h, sizeof(h), cudaMemcpyHostToDevice, c->stream));
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  return ODY_OK;
}

// checkpoint layout: header, DevScaler, then per local tensor in index
// order: master, state1 (if any), state2 (if any), all float32
struct CkptHeader {
  char magic[8];
  int32_t version;
  int32_t optimizer;
  int32_t ntensors_local;
  int32_t nstates;
  int64_t total_elems;
};

extern "C" int ody_ctx_export(ody_ctx* c, void* buf, size_t* bytes) {
  if (!c || !bytes) return fail(ODY_ERR_ARG, "null argument");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  const int nstates = (c->s1 ? 1 : 0) + (c->s2 ? 1 : 0);
  int64_t elems = 0;
  for (auto& d : c->tdesc) elems += d.numel;
  const size_t need = sizeof(CkptHeader) + sizeof(DevScaler) + (size_t)elems * 4 * (1 + nstates);
  if (!buf) {
    *bytes = need;
    return ODY_OK;
  }
  if (*bytes < need) return ctx_fail(c, ODY_ERR_SHAPE, "checkpoint buffer too small");
  CkptHeader h;
  memset(&h, 0, sizeof(h));
  memcpy(h.magic, "ODYMP01", 8);
  h.version = 1;
  h.optimizer = c->cfg.optimizer;
  h.ntensors_local = (int32_t)c->tdesc.size();
  h.nstates = nstates;
  h.total_elems = elems;
  uint8_t* p = (uint8_t*)buf;
  memcpy(p, &h, sizeof(h));
  p += sizeof(h);
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  ODY_CUDA(cudaMemcpyAsync(p, c->scaler, sizeof(DevScaler), cudaMemcpyDeviceToHost, c->stream));
  p += sizeof(DevScaler);
  float* arenas[3] = {c->master, c->s1, c->s2};
  for (auto& d : c->tdesc)
    for (int k = 0; k < 3; k++) {
      if (!arenas[k]) continue;
      ODY_CUDA(cudaMemcpyAsync(p, arenas[k] + d.off, (size_t)d.numel * 4, cudaMemcpyDeviceToHost, c->stream));
      p += (size_t)d.numel * 4;
    }
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  *bytes = need;
  return ODY_OK;
}

extern "C" int ody_ctx_import(ody_ctx* c, const void* buf, size_t bytes) {
  if (!c || !buf) return fail(ODY_ERR_ARG, "null argument");
  if (!c->finalized) return ctx_fail(c, ODY_ERR_STATE, "context not finalized");
  size_t need = 0;
  int rc = ody_ctx_export(c, nullptr, &need);
  if (rc) return rc;
  CkptHeader h;
  if (bytes < sizeof(h)) return ctx_fail(c, ODY_ERR_SHAPE, "checkpoint truncated");
  memcpy(&h, buf, sizeof(h));
  if (memcmp(h.magic, "ODYMP01", 8) != 0 || h.version != 1)
    return ctx_fail(c, ODY_ERR_ARG, "not an odyssey_mp checkpoint");
  if (bytes != need || h.optimizer != c->cfg.optimizer || h.ntensors_local != (int32_t)c->tdesc.size())
    return ctx_fail(c, ODY_ERR_SHAPE, "checkpoint does not match this context");
  const uint8_t* p = (const uint8_t*)buf + sizeof(h);
  ODY_CUDA(cudaSetDevice(c->cfg.device));
  ODY_CUDA(cudaMemcpyAsync(c->scaler, p, sizeof(DevScaler), cudaMemcpyHostToDevice, c->stream));
  p += sizeof(DevScaler);
  float* arenas[3] = {c->master, c->s1, c->s2};
  for (auto& d : c->tdesc)
    for (int k = 0; k < 3; k++) {
      if (!arenas[k]) continue;
      ODY_CUDA(cudaMemcpyAsync(arenas[k] + d.off, p, (size_t)d.numel * 4, cudaMemcpyHostToDevice, c->stream));
      p += (size_t)d.numel * 4;
    }
  ODY_CUDA(cudaStreamSynchronize(c->stream));
  return ODY_OK;
}

extern "C" void ody_ctx_destroy(ody_ctx* c) {
  if (!c) return;
  if (c->finalized || c->stream) cudaSetDevice(c->cfg.device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->comm) {
    std::string why;
    NcclApi* api = nccl_api(why);
    if (api) api->commDestroy(c->comm);
  }
  void* bufs[] = {c->master, c->s1, c->s2, c->grad, c->qout, c->qscale, c->amax, c->d_chunks_upd,
                  c->d_jobs, c->sync, c->d_tdesc, c->partials, c->ticket, c->scaler, c->dec,
                  c->local_stats, c->gathered};
  for (void* b : bufs)
    if (b) cudaFree(b);
  for (auto& e : c->tev) cudaEventDestroy(e);
  if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
  if (c->grad_slot[1]) cudaFree(c->grad_slot[1]);
  for (int s = 0; s < 2; s++) {
    if (c->slot_read[s]) cudaEventDestroy(c->slot_read[s]);
    if (c->slot_filled[s]) cudaEventDestroy(c->slot_filled[s]);
  }
  if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
  drop_graph(c);
  dp_release(c);
  if (c->h_dec) cudaFreeHost(c->h_dec);
  if (c->done) cudaEventDestroy(c->done);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

// ---------------------------------------------------------------------------
// Stateless single operations.  Each pointer may be host or device memory;
// host operands are staged through temporary device buffers on the calling
// thread's default stream.
// ---------------------------------------------------------------------------
// Device memory usable by this call's kernels: managed memory, or device
// memory of the calling thread's current GPU.  Another GPU's memory is not
// (without peer access a kernel reading it faults): device_elsewhere() names
// that case so the caller can refuse it before any launch.
static int device_of(const void* p) {
  if (!p) return -1;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (a.type == cudaMemoryTypeManaged) return INT32_MAX;  // reachable from every GPU
  return a.type == cudaMemoryTypeDevice ? a.device : -1;
}

static bool is_device_ptr(const void* p) {
  const int d = device_of(p);
  if (d < 0) return false;
  if (d == INT32_MAX) return true;
  int cur = 0;
  cudaGetDevice(&cur);
  return d == cur;
}

static bool device_elsewhere(const void* p) {
  const int d = device_of(p);
  return d >= 0 && d != INT32_MAX && !is_device_ptr(p);
}

namespace {
struct Staged {
  void* user = nullptr;
  void* dev = nullptr;
  size_t bytes = 0;
  bool owned = false;
};

struct Scope {
  cudaStream_t st = cudaStreamPerThread;
  std::vector<Staged> bufs;
  ~Scope() {
    for (auto& b : bufs)
      if (b.owned && b.dev) cudaFreeAsync(b.dev, st);
  }
  // in: copy host data to device; out-only: allocate
  cudaError_t stage(const void* user, size_t bytes, bool copy_in, void** dev) {
    if (!user) {
      *dev = nullptr;
      return cudaSuccess;
    }
    if (device_elsewhere(user)) return cudaErrorInvalidDevice;
    if (is_device_ptr(user)) {
      *dev = const_cast<void*>(user);
      bufs.push_back({const_cast<void*>(user), *dev, bytes, false});
      return cudaSuccess;
    }
    void* d = nullptr;
    cudaError_t e = cudaMallocAsync(&d, bytes < 16 ? 16 : bytes, st);
    if (e != cudaSuccess) return e;
    if (copy_in) {
      e = cudaMemcpyAsync(d, user, bytes, cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) return e;
    }
    bufs.push_back({const_cast<void*>(user), d, bytes, true});
    *dev = d;
    return cudaSuccess;
  }
  cudaError_t copy_out(void* user) {
    for (auto& b : bufs)
      if (b.user == user && b.owned) return cudaMemcpyAsync(user, b.dev, b.bytes, cudaMemcpyDeviceToHost, st);
    return cudaSuccess;
  }
};
}  // namespace

#define ODY_STAGE(S, ptr, bytes, in, dev)                                             \
  do {                                                                                \
    cudaError_t se_ = (S).stage((ptr), (bytes), (in), (void**)(dev));                 \
    if (se_ == cudaErrorInvalidDevice)                                                \
      return fail(ODY_ERR_ARG, "a buffer is device memory of another GPU than the current one"); \
    if (se_ != cudaSuccess)                                                           \
      return fail(ODY_ERR_CUDA, std::string("staging a buffer: ") + cudaGetErrorString(se_)); \
  } while (0)

static int check_dtype(int dt) {
  if (dt < DT_F32 || dt > DT_BF16) return fail(ODY_ERR_DTYPE, "unsupported dtype " + std::to_string(dt));
  return ODY_OK;
}

static void current_device_tables() {
  int dev = 0;
  cudaGetDevice(&dev);
  upload_fp4_tables(dev);
}

extern "C" int ody_unscale(const void* g, int32_t dt, int64_t n, float scale, void* out) {
  if (check_dtype(dt)) return ODY_ERR_DTYPE;
  if (n <= 0) return fail(ODY_ERR_SHAPE, "Cannot unscale empty gradient tensor");
  if (scale == 0.0f) return fail(ODY_ERR_ARG, "Cannot unscale with zero scale factor");
  if (!g || !out) return fail(ODY_ERR_ARG, "null pointer");
  Scope S;
  void *dg, *dout;
  const size_t b = (size_t)n * dtype_size(dt);
  ODY_STAGE(S, g, b, true, &dg);
  ODY_STAGE(S, out, b, false, &dout);
  ODY_CUDA(launch_unscale(dt, dg, n, scale, dout, S.st));
  ODY_CUDA(S.copy_out(out));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  return ODY_OK;
}

extern "C" int ody_check_finite(const void* g, int32_t dt, int64_t n, int32_t* finite) {
  if (check_dtype(dt)) return ODY_ERR_DTYPE;
  if (!finite || (!g && n > 0) || n < 0) return fail(ODY_ERR_ARG, "bad argument");
  if (n == 0) {
    *finite = 1;
    return ODY_OK;
  }
  Scope S;
  void *dg, *dc;
  ODY_STAGE(S, g, (size_t)n * dtype_size(dt), true, &dg);
  unsigned long long hc = 0;
  ODY_CUDA(cudaMallocAsync(&dc, 8, S.st));
  S.bufs.push_back({nullptr, dc, 8, true});
  ODY_CUDA(cudaMemsetAsync(dc, 0, 8, S.st));
  ODY_CUDA(launch_count_nonfinite(dt, dg, n, (unsigned long long*)dc, S.st));
  ODY_CUDA(cudaMemcpyAsync(&hc, dc, 8, cudaMemcpyDeviceToHost, S.st));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  *finite = hc == 0;
  return ODY_OK;
}

extern "C" int ody_to_fp32(const void* x, int32_t dt, int64_t n, float* out) {
  if (check_dtype(dt)) return ODY_ERR_DTYPE;
  if (n <= 0) return fail(ODY_ERR_SHAPE, "Cannot convert empty parameter tensor");
  if (!x || !out) return fail(ODY_ERR_ARG, "null pointer");
  Scope S;
  void *dx, *dout;
  ODY_STAGE(S, x, (size_t)n * dtype_size(dt), true, &dx);
  ODY_STAGE(S, out, (size_t)n * 4, false, &dout);
  // upcast = dequantise of the FP16/BF16 kinds; float32 is a copy
  if (dt == DT_F32)
    ODY_CUDA(cudaMemcpyAsync(dout, dx, (size_t)n * 4, cudaMemcpyDeviceToDevice, S.st));
  else
    ODY_CUDA(launch_dequantize(dt == DT_F16 ? Q_FP16 : Q_BF16, (const uint8_t*)dx, n, nullptr, (float*)dout, S.st));
  ODY_CUDA(S.copy_out(out));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  return ODY_OK;
}

extern "C" int ody_global_norm_clip(float* const* grads, const int64_t* numels, int32_t nt, float max_norm,
                                    float* total_norm) {
  if (!(max_norm > 0.0f)) return fail(ODY_ERR_ARG, "max_norm must be positive, got: " + std::to_string(max_norm));
  if (nt < 0 || (nt > 0 && (!grads || !numels))) return fail(ODY_ERR_ARG, "bad argument");
  Scope S;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = stats_grid(dev);
  void *part, *ticket, *tot, *norm, *coef;
  ODY_CUDA(cudaMallocAsync(&part, sizeof(StatsPartial) * grid, S.st));
  S.bufs.push_back({nullptr, part, 0, true});
  ODY_CUDA(cudaMallocAsync(&ticket, 4, S.st));
  S.bufs.push_back({nullptr, ticket, 0, true});
  ODY_CUDA(cudaMallocAsync(&tot, 8, S.st));
  S.bufs.push_back({nullptr, tot, 0, true});
  ODY_CUDA(cudaMallocAsync(&norm, 8, S.st));
  S.bufs.push_back({nullptr, norm, 0, true});
  coef = (float*)norm + 1;
  ODY_CUDA(cudaMemsetAsync(ticket, 0, 4, S.st));
  ODY_CUDA(cudaMemsetAsync(tot, 0, 8, S.st));
  std::vector<void*> dptr(nt);
  for (int i = 0; i < nt; i++) {
    if (numels[i] < 0 || (numels[i] > 0 && !grads[i])) return fail(ODY_ERR_ARG, "bad tensor");
    ODY_STAGE(S, grads[i], (size_t)numels[i] * 4, true, &dptr[i]);
    if (numels[i] > 0)
      ODY_CUDA(launch_sumsq((const float*)dptr[i], numels[i], (StatsPartial*)part, grid, (unsigned*)ticket,
                            (double*)tot, S.st));
  }
  ODY_CUDA(launch_clip_coef((const double*)tot, max_norm, (float*)norm, (float*)coef, S.st));
  for (int i = 0; i < nt; i++)
    if (numels[i] > 0) ODY_CUDA(launch_scale_inplace((float*)dptr[i], numels[i], (const float*)coef, S.st));
  for (int i = 0; i < nt; i++) ODY_CUDA(S.copy_out(grads[i]));
  float hn = 0.0f;
  ODY_CUDA(cudaMemcpyAsync(&hn, norm, 4, cudaMemcpyDeviceToHost, S.st));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  if (total_norm) *total_norm = hn;
  return ODY_OK;
}

extern "C" int ody_clip_global_norm_variant(float* const* grads, const int64_t* numels, int32_t nt,
                                            double max_norm, int32_t mode, double* total_norm) {
  if (mode != 0 && mode != 1) return fail(ODY_ERR_ARG, "mode must be 0 or 1");
  if (max_norm < 0.0) {
    char buf[64];
    snprintf(buf, sizeof(buf), "%g", max_norm);
    return fail(ODY_ERR_ARG, std::string("max_norm must be non-negative, got: ") + buf);
  }
  if (nt <= 0) return fail(ODY_ERR_ARG, mode == 0 ? "grads list cannot be empty" : "tensors list cannot be empty");
  if (!grads || !numels) return fail(ODY_ERR_ARG, "bad argument");
  Scope S;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = stats_grid(dev);
  void *part, *ticket, *tot;
  ODY_CUDA(cudaMallocAsync(&part, sizeof(StatsPartial) * grid, S.st));
  S.bufs.push_back({nullptr, part, 0, true});
  ODY_CUDA(cudaMallocAsync(&ticket, 4, S.st));
  S.bufs.push_back({nullptr, ticket, 0, true});
  ODY_CUDA(cudaMallocAsync(&tot, 32, S.st));  // total, norm, coef[2]
  S.bufs.push_back({nullptr, tot, 0, true});
  double* dtot = (double*)tot;
  ODY_CUDA(cudaMemsetAsync(ticket, 0, 4, S.st));
  ODY_CUDA(cudaMemsetAsync(tot, 0, 32, S.st));
  std::vector<void*> dptr(nt);
  for (int i = 0; i < nt; i++) {
    if (numels[i] < 0 || (numels[i] > 0 && !grads[i])) return fail(ODY_ERR_ARG, "bad tensor");
    ODY_STAGE(S, grads[i], (size_t)numels[i] * 4, true, &dptr[i]);
    if (numels[i] > 0) {
      if (mode == 0)
        ODY_CUDA(launch_sumsq((const float*)dptr[i], numels[i], (StatsPartial*)part, grid, (unsigned*)ticket, dtot,
                              S.st));
      else
        ODY_CUDA(launch_sumsq64((const float*)dptr[i], numels[i], (StatsPartial*)part, grid, (unsigned*)ticket,
                                dtot, S.st));
    }
  }
  ODY_CUDA(launch_clip_variant_coef(dtot, max_norm, dtot + 1, dtot + 2, S.st));
  for (int i = 0; i < nt; i++)
    if (numels[i] > 0) ODY_CUDA(launch_clip_variant_scale((float*)dptr[i], numels[i], dtot + 2, mode, S.st));
  for (int i = 0; i < nt; i++) ODY_CUDA(S.copy_out(grads[i]));
  double hn = 0.0;
  ODY_CUDA(cudaMemcpyAsync(&hn, dtot + 1, 8, cudaMemcpyDeviceToHost, S.st));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  if (total_norm) *total_norm = hn;
  return ODY_OK;
}

static int opt_common(int opt, const float* p, const float* g, const float* s1, const float* s2, int64_t n,
                      int64_t t, double lr, double mu, double b1, double b2, double eps, double wd, float* op,
                      float* os1, float* os2, double alpha = 0.99) {
  if (n <= 0) return fail(ODY_ERR_SHAPE, "Parameters and gradients must have the same shape");
  if (!p || !g || !op) return fail(ODY_ERR_ARG, "null pointer");
  if (opt == OPT_SGD) {
    if (mu > 0.0 && !s1)
      return fail(ODY_ERR_ARG, "Velocity buffer required when using momentum (use zeros_like(params))");
  } else if (opt == OPT_LION) {
    if (!s1 || !os1) return fail(ODY_ERR_ARG, "lion_step: params and momentum must have the same shape");
  } else if (opt == OPT_RMSPROP) {
    if (!s1 || !os1) return fail(ODY_ERR_ARG, "square_avg must be initialized (use zeros_like(params))");
    if (t <= 0) return fail(ODY_ERR_ARG, "Timestep t must be positive (starts at 1)");
    if (mu > 0.0 && !os2) return fail(ODY_ERR_ARG, "momentum > 0 needs an output momentum buffer");
  } else if (opt == OPT_ADAGRAD) {
    if (!s1 || !os1) return fail(ODY_ERR_ARG, "accumulator must be initialized (use zeros_like(params))");
  } else {
    if (!s1 || !s2 || !os1 || !os2)
      return fail(ODY_ERR_ARG, "Moment buffers (m and v) must be initialized (use zeros_like(params))");
    if (t <= 0) return fail(ODY_ERR_ARG, "Timestep t must be positive (starts at 1)");
  }
  if (opt == OPT_RMSPROP && !(mu > 0.0)) {
    s2 = nullptr;  // no momentum buffer is read or written
    os2 = nullptr;
  }
  ody_config cfg;
  ody_config_default(&cfg);
  cfg.optimizer = opt;
  cfg.alpha = alpha;
  cfg.learning_rate = lr;
  cfg.momentum = mu;
  cfg.beta1 = b1;
  cfg.beta2 = b2;
  cfg.epsilon = eps;
  cfg.weight_decay = wd;
  const OptConsts oc = make_consts(cfg, t);
  Scope S;
  const size_t b = (size_t)n * 4;
  void *dp, *dg, *ds1 = nullptr, *ds2 = nullptr, *dop, *dos1 = nullptr, *dos2 = nullptr;
  ODY_STAGE(S, p, b, true, &dp);
  ODY_STAGE(S, g, b, true, &dg);
  if (s1) ODY_STAGE(S, s1, b, true, &ds1);
  if (s2) ODY_STAGE(S, s2, b, true, &ds2);
  ODY_STAGE(S, op, b, false, &dop);
  if (os1) ODY_STAGE(S, os1, b, false, &dos1);
  if (os2) ODY_STAGE(S, os2, b, false, &dos2);
  // SGD without a velocity input but with an output: velocity stays zero
  if (opt == OPT_SGD && !s1 && dos1) ODY_CUDA(cudaMemsetAsync(dos1, 0, b, S.st));
  ODY_CUDA(launch_opt_step(opt, oc, (const float*)dp, (const float*)dg, (const float*)ds1, (const float*)ds2, n,
                           (float*)dop, (opt == OPT_SGD && !s1) ? nullptr : (float*)dos1, (float*)dos2, S.st));
  ODY_CUDA(S.copy_out(op));
  if (os1) ODY_CUDA(S.copy_out(os1));
  if (os2) ODY_CUDA(S.copy_out(os2));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  return ODY_OK;
}

extern "C" int ody_sgd_step(const float* p, const float* g, const float* vel, int64_t n, double lr, double mu,
                            double wd, float* op, float* ov) {
  return opt_common(OPT_SGD, p, g, vel, nullptr, n, 0, lr, mu, 0.9, 0.999, 1e-8, wd, op, ov, nullptr);
}

extern "C" int ody_adam_step(const float* p, const float* g, const float* m, const float* v, int64_t n, int64_t t,
                             double lr, double b1, double b2, double eps, double wd, float* op, float* om,
                             float* ov) {
  return opt_common(OPT_ADAM, p, g, m, v, n, t, lr, 0.0, b1, b2, eps, wd, op, om, ov);
}

extern "C" int ody_adamw_step(const float* p, const float* g, const float* m, const float* v, int64_t n, int64_t t,
                              double lr, double b1, double b2, double eps, double wd, float* op, float* om,
                              float* ov) {
  return opt_common(OPT_ADAMW, p, g, m, v, n, t, lr, 0.0, b1, b2, eps, wd, op, om, ov);
}

extern "C" int ody_lion_step(const float* p, const float* g, const float* m, int64_t n, double lr, double b1,
                             double b2, double wd, float* op, float* om) {
  return opt_common(OPT_LION, p, g, m, nullptr, n, 0, lr, 0.0, b1, b2, 1e-8, wd, op, om, nullptr);
}

extern "C" int ody_rmsprop_step(const float* p, const float* g, const float* sq, const float* buf, int64_t n,
                                int64_t t, double lr, double alpha, double eps, double wd, double mu, float* op,
                                float* osq, float* obuf) {
  return opt_common(OPT_RMSPROP, p, g, sq, buf, n, t, lr, mu, 0.9, 0.999, eps, wd, op, osq, obuf, alpha);
}

extern "C" int ody_adagrad_step(const float* p, const float* g, const float* acc, int64_t n, double lr, double eps,
                                double wd, float* op, float* oacc) {
  return opt_common(OPT_ADAGRAD, p, g, acc, nullptr, n, 0, lr, 0.0, 0.9, 0.999, eps, wd, op, oacc, nullptr);
}

extern "C" int ody_quantize(int32_t kind, const void* src, int32_t sdt, int64_t n, void* out, float* ts) {
  if (kind <= ODY_Q_NONE || kind > ODY_Q_MXFP4_OCP)
    return fail(ODY_ERR_ARG, "unknown quantisation kind " + std::to_string(kind));
  if (sdt != DT_F32 && sdt != DT_BF16) return fail(ODY_ERR_DTYPE, "quantize source must be float32 or bfloat16");
  if (n <= 0) return fail(ODY_ERR_SHAPE, "cannot quantize an empty tensor");
  if (!src || !out) return fail(ODY_ERR_ARG, "null pointer");
  current_device_tables();
  Scope S;
  void *dx, *dout, *damax, *dts;
  const int64_t qb = ody_quant_bytes(kind, n);
  ODY_STAGE(S, src, (size_t)n * dtype_size(sdt), true, &dx);
  ODY_STAGE(S, out, (size_t)qb, false, &dout);
  // [0] amax bits, [1] smallest nonzero magnitude bits, [2] the tensor scale
  ODY_CUDA(cudaMallocAsync(&damax, 16, S.st));
  S.bufs.push_back({nullptr, damax, 0, true});
  dts = (uint32_t*)damax + 2;
  ODY_CUDA(cudaMemsetAsync(damax, 0, 16, S.st));
  ODY_CUDA(cudaMemsetAsync((uint32_t*)damax + 1, 0xFF, 4, S.st));
  if (kind == ODY_Q_NVFP4_TENSOR || kind == ODY_Q_FP8_E4M3_TENSOR)
    ODY_CUDA(launch_amax(sdt, dx, n, (uint32_t*)damax, S.st));
  ODY_CUDA(launch_quantize(kind, sdt, dx, n, (uint8_t*)dout, (const uint32_t*)damax, (float*)dts, S.st));
  ODY_CUDA(S.copy_out(out));
  float hts = 1.0f;
  ODY_CUDA(cudaMemcpyAsync(&hts, dts, 4, cudaMemcpyDeviceToHost, S.st));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  if (ts) *ts = hts;
  return ODY_OK;
}

extern "C" int ody_quantize_on_stream(int32_t kind, const void* src, int32_t sdt, int64_t n, void* out,
                                      float* tensor_scale, uint32_t* amax_scratch, void* stream) {
  if (kind <= ODY_Q_NONE || kind > ODY_Q_MXFP4_OCP)
    return fail(ODY_ERR_ARG, "unknown quantisation kind " + std::to_string(kind));
  if (sdt != DT_F32 && sdt != DT_BF16) return fail(ODY_ERR_DTYPE, "quantize source must be float32 or bfloat16");
  if (n <= 0) return fail(ODY_ERR_SHAPE, "cannot quantize an empty tensor");
  if (!src || !out) return fail(ODY_ERR_ARG, "null pointer");
  const bool scaled = kind == ODY_Q_NVFP4_TENSOR || kind == ODY_Q_FP8_E4M3_TENSOR;
  if (scaled && (!tensor_scale || !amax_scratch))
    return fail(ODY_ERR_ARG, "per-tensor-scaled kinds need tensor_scale and amax_scratch");
  if (!is_device_ptr(src) || !is_device_ptr(out) || (tensor_scale && !is_device_ptr(tensor_scale)) ||
      (amax_scratch && !is_device_ptr(amax_scratch)))
    return fail(ODY_ERR_ARG, "ody_quantize_on_stream takes device memory only");
  current_device_tables();
  cudaStream_t st = (cudaStream_t)stream;
  if (scaled) {
    ODY_CUDA(cudaMemsetAsync(amax_scratch, 0, 4, st));
    ODY_CUDA(cudaMemsetAsync(amax_scratch + 1, 0xFF, 4, st));
    ODY_CUDA(launch_amax(sdt, src, n, amax_scratch, st));
  }
  ODY_CUDA(launch_quantize(kind, sdt, src, n, (uint8_t*)out, scaled ? amax_scratch : nullptr,
                           scaled ? tensor_scale : nullptr, st));
  return ODY_OK;
}

extern "C" int ody_dequantize_on_stream(int32_t kind, const void* q, int64_t n, const float* tensor_scale,
                                        float* out, void* stream) {
  if (kind <= ODY_Q_NONE || kind > ODY_Q_MXFP4_OCP)
    return fail(ODY_ERR_ARG, "unknown quantisation kind " + std::to_string(kind));
  if (n <= 0) return fail(ODY_ERR_SHAPE, "cannot dequantize an empty tensor");
  if (!q || !out) return fail(ODY_ERR_ARG, "null pointer");
  if (!is_device_ptr(q) || !is_device_ptr(out) || (tensor_scale && !is_device_ptr(tensor_scale)))
    return fail(ODY_ERR_ARG, "ody_dequantize_on_stream takes device memory only");
  ODY_CUDA(launch_dequantize(kind, (const uint8_t*)q, n, tensor_scale, out, (cudaStream_t)stream));
  return ODY_OK;
}

extern "C" int ody_dequantize(int32_t kind, const void* q, int64_t n, float ts, float* out) {
  if (kind <= ODY_Q_NONE || kind > ODY_Q_MXFP4_OCP)
    return fail(ODY_ERR_ARG, "unknown quantisation kind " + std::to_string(kind));
  if (n <= 0) return fail(ODY_ERR_SHAPE, "cannot dequantize an empty tensor");
  if (!q || !out) return fail(ODY_ERR_ARG, "null pointer");
  Scope S;
  void *dq, *dout, *dts;
  ODY_STAGE(S, q, (size_t)ody_quant_bytes(kind, n), true, &dq);
  ODY_STAGE(S, out, (size_t)n * 4, false, &dout);
  ODY_CUDA(cudaMallocAsync(&dts, 4, S.st));
  S.bufs.push_back({nullptr, dts, 0, true});
  ODY_CUDA(cudaMemcpyAsync(dts, &ts, 4, cudaMemcpyHostToDevice, S.st));
  ODY_CUDA(launch_dequantize(kind, (const uint8_t*)dq, n, (const float*)dts, (float*)dout, S.st));
  ODY_CUDA(S.copy_out(out));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  return ODY_OK;
}

extern "C" int ody_fp4_single_encode(int32_t kind, const float* x, int64_t n, const uint64_t* seeds,
                                     uint8_t* values, uint8_t* scales) {
  if (kind != ODY_Q_MXFP4 && kind != ODY_Q_NVFP4)
    return fail(ODY_ERR_ARG, "FP4 singles are ODY_Q_MXFP4 or ODY_Q_NVFP4, not " + std::to_string(kind));
  if (n <= 0) return fail(ODY_ERR_SHAPE, "cannot convert an empty tensor");
  if (!x || !values || !scales) return fail(ODY_ERR_ARG, "null pointer");
  Scope S;
  void *dx, *dseeds = nullptr, *dv, *ds;
  ODY_STAGE(S, x, (size_t)n * 4, true, &dx);
  if (seeds) ODY_STAGE(S, seeds, (size_t)n * 8, true, &dseeds);
  ODY_STAGE(S, values, (size_t)n, false, &dv);
  ODY_STAGE(S, scales, (size_t)n, false, &ds);
  ODY_CUDA(launch_fp4_single_encode(kind == ODY_Q_MXFP4, (const float*)dx, n, (const uint64_t*)dseeds,
                                    (uint8_t*)dv, (uint8_t*)ds, S.st));
  ODY_CUDA(S.copy_out(values));
  ODY_CUDA(S.copy_out(scales));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  return ODY_OK;
}

extern "C" int ody_fp4_single_decode(int32_t kind, const uint8_t* values, const uint8_t* scales, int64_t n,
                                     float* out) {
  if (kind != ODY_Q_MXFP4 && kind != ODY_Q_NVFP4)
    return fail(ODY_ERR_ARG, "FP4 singles are ODY_Q_MXFP4 or ODY_Q_NVFP4, not " + std::to_string(kind));
  if (n <= 0) return fail(ODY_ERR_SHAPE, "cannot convert an empty tensor");
  if (!values || !scales || !out) return fail(ODY_ERR_ARG, "null pointer");
  Scope S;
  void *dv, *ds, *dout;
  ODY_STAGE(S, values, (size_t)n, true, &dv);
  ODY_STAGE(S, scales, (size_t)n, true, &ds);
  ODY_STAGE(S, out, (size_t)n * 4, false, &dout);
  ODY_CUDA(launch_fp4_single_decode(kind == ODY_Q_MXFP4, (const uint8_t*)dv, (const uint8_t*)ds, n,
                                    (float*)dout, S.st));
  ODY_CUDA(S.copy_out(out));
  ODY_CUDA(cudaStreamSynchronize(S.st));
  return ODY_OK;
}

// per-format entry points over ody_quantize / ody_dequantize
extern "C" int ody_quant_mxfp4(const void* src, int32_t sdt, int64_t n, void* out) {
  return ody_quantize(ODY_Q_MXFP4, src, sdt, n, out, nullptr);
}
extern "C" int ody_dequant_mxfp4(const void* q, int64_t n, float* out) {
  return ody_dequantize(ODY_Q_MXFP4, q, n, 1.0f, out);
}
extern "C" int ody_quant_nvfp4(const void* src, int32_t sdt, int64_t n, void* out) {
  return ody_quantize(ODY_Q_NVFP4, src, sdt, n, out, nullptr);
}
extern "C" int ody_dequant_nvfp4(const void* q, int64_t n, float* out) {
  return ody_dequantize(ODY_Q_NVFP4, q, n, 1.0f, out);
}
extern "C" int ody_quant_fp8_e4m3(const void* src, int32_t sdt, int64_t n, void* out) {
  return ody_quantize(ODY_Q_FP8_E4M3, src, sdt, n, out, nullptr);
}
extern "C" int ody_dequant_fp8_e4m3(const void* q, int64_t n, float* out) {
  return ody_dequantize(ODY_Q_FP8_E4M3, q, n, 1.0f, out);
}
extern "C" int ody_quant_fp8_e5m2(const void* src, int32_t sdt, int64_t n, void* out) {
  return ody_quantize(ODY_Q_FP8_E5M2, src, sdt, n, out, nullptr);
}
extern "C" int ody_dequant_fp8_e5m2(const void* q, int64_t n, float* out) {
  return ody_dequantize(ODY_Q_FP8_E5M2, q, n, 1.0f, out);
}
extern "C" int ody_quant_fp16(const void* src, int32_t sdt, int64_t n, void* out) {
  return ody_quantize(ODY_Q_FP16, src, sdt, n, out, nullptr);
}
extern "C" int ody_dequant_fp16(const void* q, int64_t n, float* out) {
  return ody_dequantize(ODY_Q_FP16, q, n, 1.0f, out);
}
extern "C" int ody_quant_bf16(const void* src, int32_t sdt, int64_t n, void* out) {
  return ody_quantize(ODY_Q_BF16, src, sdt, n, out, nullptr);
}
extern "C" int ody_dequant_bf16(const void* q, int64_t n, float* out) {
  return ody_dequantize(ODY_Q_BF16, q, n, 1.0f, out);
}

// Test hook (not part of include/odyssey_mp.h): the exact-division shortcut
// used by the per-tensor-scaled requant against IEEE division, on device
// arrays of n (x, s) pairs.
extern "C" int odyx_selftest_divide(const float* x, const float* s, int64_t n, float* fast, float* ieee) {
  ODY_CUDA(launch_selftest_divide(x, s, n, fast, ieee, cudaStreamPerThread));
  ODY_CUDA(cudaStreamSynchronize(cudaStreamPerThread));
  return ODY_OK;
}

void ody::record_error(const std::string& msg) { g_err = msg; }
