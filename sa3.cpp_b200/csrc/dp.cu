// dp.cu -- data-parallel adapter training across GPUs: the in-place sum of the flat adapter
// gradient buffer over all ranks (NCCL, on the context's stream), followed on every rank by the
// same averaged + clipped AdamW update.
//
// The reference trains on one device and accumulates per-sample gradients on the host before
// train_average_and_clip (src/train_loop.h:147-171) and AdamW (src/train_optimizer.h:42-65);
// across ranks the accumulation becomes an all-reduce (sum) and the average divides by
// samples-per-rank x ranks, so every rank applies the identical update.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or SA3K_NCCL_LIBRARY): the library keeps
// loading on machines without it, and inside a PyTorch process it binds to the NCCL that torch
// already loaded.
#include "../../include/sa3k.h"
#include "sa3k_internal.h"

#include <dlfcn.h>
#include <nccl.h>

#include <time.h>
#include <unistd.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

namespace {

struct NcclApi {
  bool loaded = false;
  std::string error;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

template <typename F>
bool bind(void* h, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

const NcclApi* nccl(std::string& err) {
  std::call_once(g_nccl_once, [] {
    const char* path = std::getenv("SA3K_NCCL_LIBRARY");
    void* h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      g_nccl.error = std::string("cannot load NCCL (libnccl.so.2 or SA3K_NCCL_LIBRARY): ") + (e ? e : "");
      return;
    }
    if (!bind(h, "ncclGetUniqueId", g_nccl.get_unique_id) ||
        !bind(h, "ncclCommInitRankConfig", g_nccl.comm_init_rank_config) ||
        !bind(h, "ncclCommGetAsyncError", g_nccl.get_async_error) || !bind(h, "ncclCommAbort", g_nccl.comm_abort) ||
        !bind(h, "ncclCommDestroy", g_nccl.comm_destroy) || !bind(h, "ncclAllReduce", g_nccl.all_reduce) ||
        !bind(h, "ncclGetErrorString", g_nccl.error_string)) {
      g_nccl.error = "the loaded NCCL library lacks a required symbol";
      return;
    }
    g_nccl.loaded = true;
  });
  if (!g_nccl.loaded) {
    err = g_nccl.error;
    return nullptr;
  }
  return &g_nccl;
}

int fail(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)len - 1);
    err[len - 1] = 0;
  }
  return 1;
}

std::string nccl_msg(const NcclApi* api, const char* what, ncclResult_t r) {
  return std::string(what) + ": " + (api->error_string ? api->error_string(r) : "NCCL error");
}

double now_s() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

// A non-blocking communicator's pending operation: poll its state until it leaves ncclInProgress
// or the deadline passes (then the caller aborts the communicator).
ncclResult_t settle(const NcclApi* api, ncclComm_t comm, double deadline) {
  ncclResult_t st = ncclInProgress;
  while (true) {
    if (api->get_async_error(comm, &st) != ncclSuccess) return ncclSystemError;
    if (st != ncclInProgress) return st;
    if (now_s() > deadline) return ncclInProgress;
    usleep(1000);
  }
}

constexpr double kInitTimeoutS = 300.0;   // sa3k_dp_comm_create's bound on the rendezvous
constexpr double kOpTimeoutS = 60.0;      // bound on enqueueing one collective

}  // namespace

struct sa3k_dp_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = 0;
};

extern "C" {

int sa3k_dp_unique_id(void* out, int out_len, char* err, int err_len) {
  if (!out || out_len < (int)sizeof(ncclUniqueId))
    return fail(err, err_len, "unique id buffer must hold 128 bytes");
  std::string e;
  const NcclApi* api = nccl(e);
  if (!api) return fail(err, err_len, e);
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return fail(err, err_len, nccl_msg(api, "ncclGetUniqueId", r));
  std::memcpy(out, &id, sizeof id);
  return 0;
}

int sa3k_dp_comm_create_timeout(sa3k_ctx* ctx, int nranks, int rank, const void* unique_id, double timeout_s,
                                sa3k_dp_comm** out, char* err, int err_len) {
  if (!ctx || !unique_id || !out) return fail(err, err_len, "NULL argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(err, err_len, "rank must be in [0, nranks)");
  if (!(timeout_s > 0.0)) return fail(err, err_len, "timeout must be positive");
  std::string e;
  const NcclApi* api = nccl(e);
  if (!api) return fail(err, err_len, e);
  if (cudaSetDevice(ctx->c.device) != cudaSuccess) return fail(err, err_len, "cudaSetDevice failed");
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof id);
  auto* c = new sa3k_dp_comm;
  c->nranks = nranks;
  c->rank = rank;
  c->device = ctx->c.device;
  // a non-blocking communicator: the rendezvous runs in the background and is polled against the
  // deadline, so a peer that never joins ends in an error here instead of a hang
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = api->comm_init_rank_config(&c->comm, nranks, id, rank, &cfg);
  if (r == ncclInProgress || r == ncclSuccess) r = c->comm ? settle(api, c->comm, now_s() + timeout_s) : r;
  if (r != ncclSuccess) {
    if (c->comm) api->comm_abort(c->comm);
    delete c;
    if (r == ncclInProgress) {
      char msg[160];
      std::snprintf(msg, sizeof msg, "ncclCommInitRankConfig: the %d ranks did not all join within %.1f s (aborted)",
                    nranks, timeout_s);
      return fail(err, err_len, msg);
    }
    return fail(err, err_len, nccl_msg(api, "ncclCommInitRankConfig", r));
  }
  *out = c;
  return 0;
}

int sa3k_dp_comm_create(sa3k_ctx* ctx, int nranks, int rank, const void* unique_id, sa3k_dp_comm** out,
                        char* err, int err_len) {
  return sa3k_dp_comm_create_timeout(ctx, nranks, rank, unique_id, kInitTimeoutS, out, err, err_len);
}

void sa3k_dp_comm_destroy(sa3k_dp_comm* comm) {
  if (!comm) return;
  std::string e;
  const NcclApi* api = nccl(e);
  if (api && comm->comm) {
    cudaSetDevice(comm->device);
    api->comm_destroy(comm->comm);
  }
  delete comm;
}

int sa3k_dp_allreduce_sum(sa3k_ctx* ctx, sa3k_dp_comm* comm, float* buf, int64_t n, char* err, int err_len) {
  if (!ctx || !comm || (!buf && n > 0)) return fail(err, err_len, "NULL argument");
  if (n < 0) return fail(err, err_len, "n must be >= 0");
  if (comm->device != ctx->c.device) return fail(err, err_len, "communicator and context are on different devices");
  if (n == 0 || comm->nranks == 1) return 0;
  std::string e;
  const NcclApi* api = nccl(e);
  if (!api) return fail(err, err_len, e);
  cudaSetDevice(ctx->c.device);
  ncclResult_t r = api->all_reduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, comm->comm, ctx->c.stream);
  if (r == ncclInProgress) r = settle(api, comm->comm, now_s() + kOpTimeoutS);   // non-blocking enqueue
  if (r == ncclInProgress) return fail(err, err_len, "ncclAllReduce: not enqueued within the time limit");
  if (r != ncclSuccess) return fail(err, err_len, nccl_msg(api, "ncclAllReduce", r));
  return 0;
}

int sa3k_dp_allreduce_adamw(sa3k_ctx* ctx, sa3k_dp_comm* comm, float* p, float* g, float* m, float* v,
                            int64_t n, int samples_per_rank, const sa3k_adamw_params* hp, int step,
                            double* grad_norm_out, char* err, int err_len) {
  if (!ctx || !comm || !p || !g || !m || !v || !hp) return fail(err, err_len, "NULL argument");
  if (samples_per_rank <= 0) return fail(err, err_len, "cannot apply empty gradient batch");
  if (sa3k_dp_allreduce_sum(ctx, comm, g, n, err, err_len)) return 1;
  return sa3k_average_clip_adamw(ctx, p, g, m, v, n, samples_per_rank * comm->nranks, hp, step, grad_norm_out,
                                 err, err_len);
}

int sa3k_dp_comm_info(const sa3k_dp_comm* comm, int* nranks, int* rank) {
  if (!comm) return 1;
  if (nranks) *nranks = comm->nranks;
  if (rank) *rank = comm->rank;
  return 0;
}

}  // extern "C"
