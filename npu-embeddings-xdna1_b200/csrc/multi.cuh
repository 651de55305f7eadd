// Several GPUs: the request batch sharded over them, the pooled rows
// gathered to the serving rank over NCCL.  Included at the end of nebw.cu
// (it drives the encoder pass defined there).
//
// Every sequence is an independent encoder pass -- the reference computes
// rows independently (gemm_nt, LayerNorm and pooling are row-local and
// attention is per (sequence, head): runtime/include/common/conv_host.hpp:
// 154-158, runtime/src/encoders/bert_encoder.cpp:1001-1004) -- so a batch
// splits across GPUs with one weight replica per GPU and no exchange on the
// data path.  The one collective is the gather of each rank's [b_r, hidden]
// fp32 rows to the root at the end of a pass (ncclSend / ncclRecv in one
// group; NVLink / NVSwitch carries it), after which a kernel on the root
// scatters the rank-major rows back into request order.  No kernel here or
// in the encoder reads another GPU's memory.
//
// The reference's only concurrency is host threads over one NPU (the
// --pipeline lanes of EmbedService::embed, runtime/src/server/
// embed_service.cpp:66-108); nebw_encode_multi is that lane structure
// recast as one host thread per GPU.
//
// NCCL is opened with dlopen("libnccl.so.2", or $NEBW_NCCL_LIB) on first
// use, so the library loads where NCCL is absent and only these entry points
// fail, by name.  In a process that already loaded NCCL (a PyTorch process),
// the loaded copy is the one used; a process that loads another NCCL later
// (by importing PyTorch after the first communicator call) would be handed
// this one by the dynamic loader, so it should load that one first.  Communicators are non-blocking, and every wait on one --
// initialisation, the enqueue of a group, the completion of a gather -- is
// bounded by the communicator's timeout; on expiry the communicator is
// aborted (ncclCommAbort ends its kernels) and the call returns NEBW_ECOMM.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <numeric>
#include <thread>

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int *) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

int nccl_api(const NcclApi **out) {
  std::call_once(g_nccl_once, [] {
    // a copy the process already holds (a PyTorch process loads its own
    // with libtorch) is the one to use: a second one would be found by
    // soname by every later loader of libnccl.so.2
    const char *path = std::getenv("NEBW_NCCL_LIB");
    if (!path || !*path) path = "libnccl.so.2";
    void *h = dlopen(path, RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char *e = dlerror();
      g_nccl.why = std::string(path) + " could not be loaded: " + (e ? e : "unknown");
      return;
    }
    bool all = true;
    auto sym = [&](auto &fn, const char *name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) {
        all = false;
        g_nccl.why += std::string(g_nccl.why.empty() ? "" : ", ") + name;
      }
    };
    sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
    sym(g_nccl.CommInitRankConfig, "ncclCommInitRankConfig");
    sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError");
    sym(g_nccl.CommAbort, "ncclCommAbort");
    sym(g_nccl.CommDestroy, "ncclCommDestroy");
    sym(g_nccl.CommFinalize, "ncclCommFinalize");
    sym(g_nccl.GroupStart, "ncclGroupStart");
    sym(g_nccl.GroupEnd, "ncclGroupEnd");
    sym(g_nccl.Send, "ncclSend");
    sym(g_nccl.Recv, "ncclRecv");
    sym(g_nccl.GetErrorString, "ncclGetErrorString");
    sym(g_nccl.GetVersion, "ncclGetVersion");
    if (!all) {
      g_nccl.why = "libnccl.so.2 lacks " + g_nccl.why;
      return;
    }
    g_nccl.ok = true;
  });
  if (!g_nccl.ok) return set_error(NEBW_ECOMM, "NCCL unavailable: %s", g_nccl.why.c_str());
  *out = &g_nccl;
  return NEBW_OK;
}

// Scatter the root's rank-major gathered rows into request order:
// out[order[k]] = rows[k], one CTA per row, float4 lanes (H % 4 == 0).
__global__ void scatter_rows_kernel(const float *__restrict__ rows, const int *__restrict__ order,
                                    int n, int H, float *__restrict__ out) {
  const int k = blockIdx.x;
  if (k >= n) return;
  const int dst = __ldg(order + k);
  const float4 *src = reinterpret_cast<const float4 *>(rows + static_cast<int64_t>(k) * H);
  float4 *d = reinterpret_cast<float4 *>(out + static_cast<int64_t>(dst) * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) d[i] = src[i];
}

}  // namespace

struct nebw_comm {
  nebw_dev *dev = nullptr;
  ncclComm_t comm = nullptr;
  int32_t nranks = 0, rank = 0;
  double timeout_s = 60.0;
  bool aborted = false;
  // device buffers, grown on demand: this rank's pooled rows, and at the
  // root the gathered rank-major rows, their request order and the result
  int64_t rows_cap = 0, batch_cap = 0, hidden = 0;
  float *shard_out = nullptr, *gathered = nullptr, *result = nullptr;
  int *order = nullptr;
  // pinned host staging of the host-buffer entry point
  int64_t ids_cap = 0, lens_cap = 0, order_cap = 0;
  int32_t *ids_pinned = nullptr, *lens_pinned = nullptr, *order_pinned = nullptr;
};

namespace {

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int comm_fail(nebw_comm *c, const char *what, const char *why) {
  const NcclApi *api = nullptr;
  if (c->comm && !c->aborted && nccl_api(&api) == NEBW_OK) api->CommAbort(c->comm);
  c->aborted = true;
  c->comm = nullptr;
  return set_error(NEBW_ECOMM, "%s (rank %d of %d): %s; the communicator was aborted", what,
                   c->rank, c->nranks, why);
}

// Wait until the communicator has no operation in progress (initialisation,
// or the enqueue of a group), for at most its timeout.
int comm_wait_ready(nebw_comm *c, const char *what) {
  const NcclApi *api = nullptr;
  if (int rc = nccl_api(&api)) return rc;
  const double deadline = now_s() + c->timeout_s;
  while (true) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = api->CommGetAsyncError(c->comm, &st);
    if (q != ncclSuccess) return comm_fail(c, what, api->GetErrorString(q));
    if (st == ncclSuccess) return NEBW_OK;
    if (st != ncclInProgress) return comm_fail(c, what, api->GetErrorString(st));
    if (now_s() > deadline) return comm_fail(c, what, "no progress within the timeout");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Wait until `st` has drained, for at most the communicator's timeout,
// watching the communicator for an asynchronous error meanwhile.
int comm_wait_stream(nebw_comm *c, cudaStream_t st, const char *what) {
  const NcclApi *api = nullptr;
  if (int rc = nccl_api(&api)) return rc;
  const double deadline = now_s() + c->timeout_s;
  while (true) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return NEBW_OK;
    if (e != cudaErrorNotReady)
      return set_error(NEBW_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    ncclResult_t as = ncclSuccess;
    api->CommGetAsyncError(c->comm, &as);
    if (as != ncclSuccess && as != ncclInProgress) return comm_fail(c, what, api->GetErrorString(as));
    if (now_s() > deadline) return comm_fail(c, what, "the stream did not drain within the timeout");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

int comm_usable(const nebw_comm *c) {
  NEBW_REQUIRE(c != nullptr, "null communicator");
  if (c->aborted || !c->comm)
    return set_error(NEBW_ESTATE, "the communicator was aborted after an earlier failure; "
                                  "destroy it and make a new one");
  return NEBW_OK;
}

ncclConfig_t nonblocking_config() {
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  return cfg;
}

void free_comm_buffers(nebw_comm *c) {
  cudaFree(c->shard_out);
  cudaFree(c->gathered);
  cudaFree(c->result);
  cudaFree(c->order);
  cudaFreeHost(c->ids_pinned);
  cudaFreeHost(c->lens_pinned);
  cudaFreeHost(c->order_pinned);
  c->shard_out = c->gathered = c->result = nullptr;
  c->order = nullptr;
  c->ids_pinned = c->lens_pinned = c->order_pinned = nullptr;
  c->rows_cap = c->batch_cap = c->ids_cap = c->lens_cap = c->order_cap = 0;
}

// Device buffers for `b_r` local rows and (at the root) a batch of B rows of
// width H.
int comm_buffers(nebw_comm *c, int64_t b_r, int64_t B, int64_t H) {
  if (H != c->hidden) {
    NEBW_CUDA(cudaStreamSynchronize(c->dev->stream));
    cudaFree(c->shard_out);
    cudaFree(c->gathered);
    cudaFree(c->result);
    c->shard_out = c->gathered = c->result = nullptr;
    c->rows_cap = c->batch_cap = 0;
    c->hidden = H;
  }
  if (b_r > c->rows_cap) {
    cudaFree(c->shard_out);
    c->shard_out = nullptr;
    if (cudaMalloc(&c->shard_out, static_cast<size_t>(std::max<int64_t>(b_r, 1) * H * 4)) != cudaSuccess) {
      cudaGetLastError();
      return set_error(NEBW_ENOMEM, "shard output of %lld rows", static_cast<long long>(b_r));
    }
    c->rows_cap = b_r;
  }
  if (c->rank == 0 && B > c->batch_cap) {
    cudaFree(c->gathered);
    cudaFree(c->result);
    cudaFree(c->order);
    c->gathered = c->result = nullptr;
    c->order = nullptr;
    const size_t rb = static_cast<size_t>(B * H * 4);
    if (cudaMalloc(&c->gathered, rb) != cudaSuccess || cudaMalloc(&c->result, rb) != cudaSuccess ||
        cudaMalloc(&c->order, static_cast<size_t>(B) * 4) != cudaSuccess) {
      cudaGetLastError();
      return set_error(NEBW_ENOMEM, "gather buffers for a batch of %lld", static_cast<long long>(B));
    }
    c->batch_cap = B;
  }
  return NEBW_OK;
}

// The gather: root receives counts[r] rows of H fp32 from each rank r into
// out_dev at rank-major offsets; the root's own rows are a device copy.
int gather_rows(nebw_comm *c, const float *rows, const int32_t *counts, int64_t H, float *out,
                int32_t root, cudaStream_t st) {
  const NcclApi *api = nullptr;
  if (int rc = nccl_api(&api)) return rc;
  std::vector<int64_t> at(static_cast<size_t>(c->nranks) + 1, 0);
  for (int r = 0; r < c->nranks; ++r) at[r + 1] = at[r] + counts[r];
  const int64_t mine = counts[c->rank];
  if (c->rank == root && mine > 0 && out + at[root] * H != rows)
    NEBW_CUDA(cudaMemcpyAsync(out + at[root] * H, rows, static_cast<size_t>(mine * H * 4),
                              cudaMemcpyDeviceToDevice, st));
  if (c->nranks == 1) return NEBW_OK;
  ncclResult_t q = api->GroupStart();
  if (q == ncclSuccess) {
    if (c->rank == root) {
      for (int r = 0; r < c->nranks && q == ncclSuccess; ++r)
        if (r != root && counts[r] > 0)
          q = api->Recv(out + at[r] * H, static_cast<size_t>(counts[r] * H), ncclFloat32, r,
                        c->comm, st);
    } else if (mine > 0) {
      q = api->Send(rows, static_cast<size_t>(mine * H), ncclFloat32, root, c->comm, st);
    }
    const ncclResult_t e = api->GroupEnd();
    if (q == ncclSuccess) q = e;
  }
  if (q != ncclSuccess && q != ncclInProgress) return comm_fail(c, "gather", api->GetErrorString(q));
  return comm_wait_ready(c, "gather enqueue");
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI: multi-GPU
// ---------------------------------------------------------------------------

extern "C" int nebw_comm_unique_id(uint8_t id[NEBW_COMM_ID_BYTES]) {
  NEBW_REQUIRE(id != nullptr, "null id buffer");
  static_assert(sizeof(ncclUniqueId) == NEBW_COMM_ID_BYTES, "NCCL unique id size");
  const NcclApi *api = nullptr;
  if (int rc = nccl_api(&api)) return rc;
  ncclUniqueId u;
  const ncclResult_t q = api->GetUniqueId(&u);
  if (q != ncclSuccess) return set_error(NEBW_ECOMM, "ncclGetUniqueId: %s", api->GetErrorString(q));
  std::memcpy(id, &u, sizeof u);
  return NEBW_OK;
}

extern "C" int nebw_comm_init_rank(nebw_dev *dev, int32_t nranks, int32_t rank,
                                   const uint8_t id[NEBW_COMM_ID_BYTES], double timeout_s,
                                   nebw_comm **out) {
  NEBW_REQUIRE(out && id, "null argument");
  *out = nullptr;
  NEBW_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "rank %d of %d refused", rank, nranks);
  NEBW_REQUIRE(timeout_s > 0.0, "timeout must be positive");
  if (int rc = use_dev(dev)) return rc;
  const NcclApi *api = nullptr;
  if (int rc = nccl_api(&api)) return rc;
  std::unique_ptr<nebw_comm> c(new nebw_comm());
  c->dev = dev;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_s = timeout_s;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof u);
  ncclConfig_t cfg = nonblocking_config();
  const ncclResult_t q = api->CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  if (q != ncclSuccess && q != ncclInProgress) {
    if (c->comm) api->CommAbort(c->comm);
    return set_error(NEBW_ECOMM, "ncclCommInitRankConfig (rank %d of %d): %s", rank, nranks,
                     api->GetErrorString(q));
  }
  if (int rc = comm_wait_ready(c.get(), "communicator initialisation")) return rc;
  *out = c.release();
  return NEBW_OK;
}

extern "C" int nebw_comm_init_all(int32_t n, nebw_dev *const *devs, double timeout_s,
                                  nebw_comm **comms) {
  NEBW_REQUIRE(n >= 1 && devs && comms, "null or empty argument");
  NEBW_REQUIRE(timeout_s > 0.0, "timeout must be positive");
  for (int i = 0; i < n; ++i) {
    comms[i] = nullptr;
    NEBW_REQUIRE(devs[i] != nullptr, "null device handle %d", i);
    for (int j = 0; j < i; ++j)
      NEBW_REQUIRE(devs[j]->device != devs[i]->device, "GPU %d given twice", devs[i]->device);
  }
  const NcclApi *api = nullptr;
  if (int rc = nccl_api(&api)) return rc;
  ncclUniqueId u;
  ncclResult_t q = api->GetUniqueId(&u);
  if (q != ncclSuccess) return set_error(NEBW_ECOMM, "ncclGetUniqueId: %s", api->GetErrorString(q));
  std::vector<std::unique_ptr<nebw_comm>> cs(static_cast<size_t>(n));
  std::vector<ncclConfig_t> cfgs(static_cast<size_t>(n), nonblocking_config());
  // one thread initialises every rank inside one group (NCCL's form for
  // several GPUs per thread)
  q = api->GroupStart();
  for (int i = 0; i < n && (q == ncclSuccess || q == ncclInProgress); ++i) {
    cs[i].reset(new nebw_comm());
    cs[i]->dev = devs[i];
    cs[i]->nranks = n;
    cs[i]->rank = i;
    cs[i]->timeout_s = timeout_s;
    if (cudaSetDevice(devs[i]->device) != cudaSuccess) {
      q = ncclUnhandledCudaError;
      break;
    }
    q = api->CommInitRankConfig(&cs[i]->comm, n, u, i, &cfgs[i]);
  }
  const ncclResult_t e = api->GroupEnd();
  if (q == ncclSuccess || q == ncclInProgress) q = e;
  int rc = NEBW_OK;
  if (q != ncclSuccess && q != ncclInProgress) {
    rc = set_error(NEBW_ECOMM, "communicator initialisation over %d GPUs: %s", n,
                   api->GetErrorString(q));
  }
  for (int i = 0; i < n && rc == NEBW_OK; ++i) {
    if (!cs[i] || !cs[i]->comm) {
      rc = set_error(NEBW_ECOMM, "communicator initialisation over %d GPUs did not create rank %d", n, i);
      break;
    }
    cudaSetDevice(devs[i]->device);
    rc = comm_wait_ready(cs[i].get(), "communicator initialisation");
  }
  if (rc != NEBW_OK) {
    for (auto &c : cs)
      if (c && c->comm && !c->aborted) api->CommAbort(c->comm);
    return rc;
  }
  for (int i = 0; i < n; ++i) comms[i] = cs[i].release();
  return NEBW_OK;
}

extern "C" int nebw_comm_destroy(nebw_comm *c) {
  if (!c) return NEBW_OK;
  cudaSetDevice(c->dev->device);
  const NcclApi *api = nullptr;
  int rc = NEBW_OK;
  if (c->comm && !c->aborted && nccl_api(&api) == NEBW_OK) {
    // finalize flushes outstanding work (bounded), then destroy frees it
    const ncclResult_t q = api->CommFinalize(c->comm);
    if (q != ncclSuccess && q != ncclInProgress) {
      rc = comm_fail(c, "communicator finalisation", api->GetErrorString(q));
    } else if ((rc = comm_wait_ready(c, "communicator finalisation")) == NEBW_OK) {
      api->CommDestroy(c->comm);
    }
  }
  free_comm_buffers(c);
  delete c;
  return rc;
}

extern "C" int nebw_comm_size(const nebw_comm *c, int32_t *nranks, int32_t *rank) {
  NEBW_REQUIRE(c && nranks && rank, "null argument");
  *nranks = c->nranks;
  *rank = c->rank;
  return NEBW_OK;
}

// Length-balanced plan: sequences in decreasing cost order (cost l + l^2 /
// 2048: the GEMMs grow with l, attention with l^2, weighted as in a
// BERT-large layer; ties by index), each to the rank with the least cost so
// far (ties to the lowest rank).
extern "C" int nebw_shard_plan(const int32_t *lens, int32_t B, int32_t nranks, int32_t *owner,
                               int32_t *counts) {
  NEBW_REQUIRE(lens && owner && counts, "null argument");
  NEBW_REQUIRE(B >= 0 && nranks >= 1, "plan of %d sequences over %d ranks refused", B, nranks);
  std::vector<double> cost(static_cast<size_t>(B));
  for (int32_t i = 0; i < B; ++i) {
    const double l = lens[i];
    cost[i] = l + l * l / 2048.0;
  }
  std::vector<int32_t> by_cost(static_cast<size_t>(B));
  std::iota(by_cost.begin(), by_cost.end(), 0);
  std::stable_sort(by_cost.begin(), by_cost.end(),
                   [&](int32_t a, int32_t b) { return cost[a] > cost[b]; });
  std::vector<double> load(static_cast<size_t>(nranks), 0.0);
  for (int32_t r = 0; r < nranks; ++r) counts[r] = 0;
  for (int32_t i : by_cost) {
    const int32_t r = static_cast<int32_t>(std::min_element(load.begin(), load.end()) - load.begin());
    owner[i] = r;
    load[r] += cost[i];
    ++counts[r];
  }
  return NEBW_OK;
}

// order[k] = the request index of gathered row k: rank-major, each rank's
// sequences ascending.
extern "C" int nebw_shard_order(const int32_t *owner, int32_t B, int32_t nranks, int32_t *order) {
  NEBW_REQUIRE(owner && order, "null argument");
  NEBW_REQUIRE(B >= 0 && nranks >= 1, "order of %d sequences over %d ranks refused", B, nranks);
  std::vector<int32_t> at(static_cast<size_t>(nranks) + 1, 0);
  for (int32_t i = 0; i < B; ++i) {
    NEBW_REQUIRE(owner[i] >= 0 && owner[i] < nranks, "owner[%d] = %d outside [0, %d)", i, owner[i],
                 nranks);
    ++at[owner[i] + 1];
  }
  for (int32_t r = 0; r < nranks; ++r) at[r + 1] += at[r];
  for (int32_t i = 0; i < B; ++i) order[at[owner[i]]++] = i;
  return NEBW_OK;
}

extern "C" int nebw_gather_rows(nebw_comm *c, const float *rows_dev, const int32_t *counts,
                                int32_t H, float *out_dev, int32_t root, void *stream) {
  if (int rc = comm_usable(c)) return rc;
  NEBW_REQUIRE(counts && H > 0 && root >= 0 && root < c->nranks, "gather arguments refused");
  NEBW_REQUIRE(c->rank != root || out_dev, "the root needs an output buffer");
  NEBW_REQUIRE(counts[c->rank] == 0 || rows_dev, "rows to send but no buffer");
  if (int rc = use_dev(c->dev)) return rc;
  return gather_rows(c, rows_dev, counts, H, out_dev, root, pick_stream(c->dev, stream));
}

extern "C" int nebw_comm_sync(nebw_comm *c, void *stream) {
  if (int rc = comm_usable(c)) return rc;
  if (int rc = use_dev(c->dev)) return rc;
  if (int rc = comm_wait_stream(c, pick_stream(c->dev, stream), "collective completion")) return rc;
  return nebw_sync(c->dev);
}

namespace {

// Encode this rank's b_r sequences (device ids / lens) into the
// communicator's shard buffer, gather to rank 0 and, at rank 0, scatter into
// request order (order_dev) or keep rank order (order_dev null) in out_dev.
int encode_gather(nebw_model *m, nebw_comm *c, const int32_t *ids_dev, const int32_t *lens_dev,
                  int32_t b_r, int32_t S, const int32_t *counts, const int32_t *order_dev,
                  float *out_dev, cudaStream_t st) {
  const int64_t H = m->cfg.hidden;
  int64_t B = 0;
  for (int r = 0; r < c->nranks; ++r) {
    NEBW_REQUIRE(counts[r] >= 0, "counts[%d] = %d refused", r, counts[r]);
    B += counts[r];
  }
  NEBW_REQUIRE(counts[c->rank] == b_r, "this rank's count %d differs from its %d sequences",
               counts[c->rank], b_r);
  NEBW_REQUIRE(B > 0, "empty batch refused");
  if (int rc = comm_buffers(c, b_r, B, H)) return rc;
  if (b_r > 0) {
    if (int rc = check_pass(m, b_r, S)) return rc;
    if (int rc = ensure_workspace(m, b_r, S)) return rc;
    if (int rc = run_pass(m, ids_dev, lens_dev, b_r, S, c->shard_out, st))
      return rc;
  }
  float *land = c->rank == 0 ? (order_dev ? c->gathered : out_dev) : nullptr;
  if (int rc = gather_rows(c, c->shard_out, counts, H, land, 0, st)) return rc;
  if (c->rank == 0 && order_dev) {
    scatter_rows_kernel<<<static_cast<unsigned>(B), 256, 0, st>>>(c->gathered, order_dev,
                                                                  static_cast<int>(B),
                                                                  static_cast<int>(H), out_dev);
    NEBW_CUDA(cudaGetLastError());
  }
  return NEBW_OK;
}

}  // namespace

extern "C" int nebw_encode_shard_gather(nebw_model *m, nebw_comm *c, const int32_t *ids_dev,
                                        const int32_t *lens_dev, int32_t b_r, int32_t S,
                                        const int32_t *counts, const int32_t *order_dev,
                                        float *out_dev, void *stream) {
  NEBW_REQUIRE(m && counts, "null argument");
  if (int rc = comm_usable(c)) return rc;
  NEBW_REQUIRE(m->dev == c->dev, "model and communicator are on different device handles");
  NEBW_REQUIRE(b_r == 0 || (ids_dev && lens_dev), "null shard buffers");
  NEBW_REQUIRE(c->rank != 0 || out_dev, "rank 0 needs an output buffer");
  if (int rc = use_dev(m->dev)) return rc;
  return encode_gather(m, c, ids_dev, lens_dev, b_r, S, counts, order_dev, out_dev,
                       pick_stream(m->dev, stream));
}

extern "C" int nebw_encode_sharded(nebw_model *m, nebw_comm *c, const int32_t *ids,
                                   const int32_t *lens, int32_t B, int32_t S, float *out) {
  NEBW_REQUIRE(m && ids && lens, "null argument");
  if (int rc = comm_usable(c)) return rc;
  NEBW_REQUIRE(m->dev == c->dev, "model and communicator are on different device handles");
  NEBW_REQUIRE(c->rank != 0 || out, "rank 0 needs an output buffer");
  NEBW_REQUIRE(B > 0 && S > 0, "empty batch refused");
  if (int rc = use_dev(m->dev)) return rc;
  nebw_dev *d = m->dev;
  cudaStream_t st = d->stream;
  const int n = c->nranks;
  std::vector<int32_t> owner(static_cast<size_t>(B)), counts(static_cast<size_t>(n));
  if (int rc = nebw_shard_plan(lens, B, n, owner.data(), counts.data())) return rc;
  const int32_t b_r = counts[c->rank];
  // pinned staging (this rank's ids and lengths, the root's order), reused
  // across calls: the previous call's copies out of it have completed
  if (int rc = comm_wait_stream(c, st, "previous sharded pass")) return rc;
  const int64_t need_ids = std::max<int64_t>(static_cast<int64_t>(b_r) * S, 1);
  if (need_ids > c->ids_cap || b_r > c->lens_cap) {
    cudaFreeHost(c->ids_pinned);
    cudaFreeHost(c->lens_pinned);
    c->ids_pinned = c->lens_pinned = nullptr;
    c->ids_cap = c->lens_cap = 0;
    const int64_t ids_cap = std::max(need_ids, c->ids_cap), lens_cap = std::max<int64_t>(b_r, 1);
    if (cudaHostAlloc(&c->ids_pinned, static_cast<size_t>(ids_cap) * 4, 0) != cudaSuccess ||
        cudaHostAlloc(&c->lens_pinned, static_cast<size_t>(lens_cap) * 4, 0) != cudaSuccess) {
      cudaGetLastError();
      return set_error(NEBW_ENOMEM, "pinned staging of the shard");
    }
    c->ids_cap = ids_cap;
    c->lens_cap = lens_cap;
  }
  for (int32_t i = 0, k = 0; i < B; ++i) {
    if (owner[i] != c->rank) continue;
    std::memcpy(c->ids_pinned + static_cast<int64_t>(k) * S, ids + static_cast<int64_t>(i) * S,
                static_cast<size_t>(S) * 4);
    c->lens_pinned[k++] = lens[i];
  }
  const int32_t *order_dev = nullptr;
  if (c->rank == 0) {
    if (B > c->order_cap) {
      cudaFreeHost(c->order_pinned);
      c->order_pinned = nullptr;
      if (cudaHostAlloc(&c->order_pinned, static_cast<size_t>(B) * 4, 0) != cudaSuccess) {
        cudaGetLastError();
        return set_error(NEBW_ENOMEM, "pinned staging of the order");
      }
      c->order_cap = B;
    }
    if (int rc = nebw_shard_order(owner.data(), B, n, c->order_pinned)) return rc;
    if (int rc = comm_buffers(c, b_r, B, m->cfg.hidden)) return rc;
    NEBW_CUDA(cudaMemcpyAsync(c->order, c->order_pinned, static_cast<size_t>(B) * 4,
                              cudaMemcpyHostToDevice, st));
    order_dev = c->order;
  }
  if (b_r > 0) {
    if (int rc = check_pass(m, b_r, S)) return rc;
    if (int rc = ensure_workspace(m, b_r, S)) return rc;
    NEBW_CUDA(cudaMemcpyAsync(m->ids, c->ids_pinned, static_cast<size_t>(b_r) * S * 4,
                              cudaMemcpyHostToDevice, st));
    NEBW_CUDA(cudaMemcpyAsync(m->len_in, c->lens_pinned, static_cast<size_t>(b_r) * 4,
                              cudaMemcpyHostToDevice, st));
  }
  if (int rc = comm_buffers(c, b_r, B, m->cfg.hidden)) return rc;
  if (int rc = encode_gather(m, c, m->ids, m->len_in, b_r, S, counts.data(), order_dev, c->result, st))
    return rc;
  if (int rc = comm_wait_stream(c, st, "sharded pass")) return rc;
  if (int rc = nebw_sync(d)) return rc;
  if (c->rank == 0)
    NEBW_CUDA(cudaMemcpy(out, c->result, static_cast<size_t>(B) * m->cfg.hidden * 4,
                         cudaMemcpyDeviceToHost));
  return NEBW_OK;
}

extern "C" int nebw_encode_multi(int32_t n, nebw_model *const *models, nebw_comm *const *comms,
                                 const int32_t *ids, const int32_t *lens, int32_t B, int32_t S,
                                 float *out) {
  NEBW_REQUIRE(n >= 1 && models && comms && ids && lens && out, "null or empty argument");
  for (int i = 0; i < n; ++i) {
    NEBW_REQUIRE(models[i] && comms[i], "null model or communicator %d", i);
    NEBW_REQUIRE(comms[i]->nranks == n && comms[i]->rank == i,
                 "communicator %d is rank %d of %d; nebw_encode_multi wants rank %d of %d", i,
                 comms[i]->rank, comms[i]->nranks, i, n);
  }
  std::vector<int> rcs(static_cast<size_t>(n), NEBW_OK);
  std::vector<std::string> msgs(static_cast<size_t>(n));
  auto lane = [&](int i) {
    rcs[i] = nebw_encode_sharded(models[i], comms[i], ids, lens, B, S, i == 0 ? out : nullptr);
    if (rcs[i]) msgs[i] = g_last_error;
  };
  std::vector<std::thread> threads;
  for (int i = 1; i < n; ++i) threads.emplace_back(lane, i);
  lane(0);
  for (auto &t : threads) t.join();
  for (int i = 0; i < n; ++i)
    if (rcs[i]) return set_error(rcs[i], "GPU lane %d: %s", i, msgs[i].c_str());
  return NEBW_OK;
}
