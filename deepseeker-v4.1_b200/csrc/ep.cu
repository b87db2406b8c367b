// Expert-parallel decode over NVLink peer memory (no collective library on
// the data path).
//
// Ranks 0..G-1 each own E/G experts of a layer and decode b tokens per step.
// One ds_ep_decode call per layer and rank:
//
//   1. ep_dispatch_kernel: every rank stores its b token rows (x, global ids,
//      gates) into slot `rank` of every rank's dispatch area (P2P stores over
//      NVLink into memory opened with CUDA IPC), then reads the G slots of
//      its own area into local buffers, rewriting the gathered ids to local
//      expert ids (-1 where another rank owns the expert).
//   2. the decode kernels (tcgen05 for FP4 banks, moe_decode_t5.cu; CUDA-core
//      for q3 banks, moe_decode_q3.cu) over the G*b gathered rows: this
//      rank's routed experts for every row and slice `rank` of the shared
//      expert's intermediate features for every row (when the shared inter
//      splits into G slices of 256; otherwise the whole shared expert for its
//      own rows), f32 partial rows out.
//   3. ep_combine_kernel: every rank stores the partial rows of rank q's
//      tokens into slot `rank` of q's combine area, then sums the G slots of
//      its own area in rank order into its bf16 output: routed partials,
//      plus the shared sum rounded to bf16 first (the reference adds the
//      shared expert's output in the activation dtype,
//      src/deepseeker/mlx_runner.py:776-781).
//
// Exchange format: every 4-byte data word travels with the call's epoch in
// one 8-byte store; a reader polls each word until it carries the epoch it
// expects, so the data needs no fence and no separate flag.  The epoch is a
// per-block counter in local device memory (every block of every rank runs
// once per call, so the counters agree); nothing is ever reset and graph
// replays keep counting.  Nothing on the path calls NCCL, so a step of many
// layers captures into one CUDA graph.  An area is written again only after
// its owner has moved past the step that reads it (a peer's next dispatch
// follows its combine, which needs this rank's combine push, which follows
// this rank's reads), so one area of each kind suffices.
//
// Every wait is bounded by %globaltimer (the communicator's timeout); a
// timeout sets the error word and an abort flag, and later kernels of an
// aborted communicator return at once.  ds_ep_status reads the error word.
//
// The per-layer call it replaces is the reference's MoE block of a decode
// step (src/deepseeker/mlx_runner.py:765-985 Runner.moe ->
// src/deepseeker/mlx_forward.py:257-419 moe_layer), here spread over ranks.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "deepseeker_b200.h"
#include "ds_common.cuh"
#include "moe_decode.cuh"
#include "ptx.cuh"

namespace {

constexpr int kMaxWorld = 8;
constexpr int kDispatchBlocks = 2;   // blocks per peer in the dispatch kernel
constexpr int kCombineBlocks = 4;    // blocks per peer in the combine kernel
constexpr int kEpThreads = 256;
constexpr int kErrTimeout = 2;

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

// Byte offsets inside one rank's region (identical on every rank).  The two
// exchange areas are written by peers in the low-latency word format (8-byte
// stores of {data word, epoch}); the rest is local.
struct EpLayout {
  size_t ll_g, ll_r;                                   // peer-written
  size_t ctr, err, recv_x, recv_w, ids_local, part, part_sh;   // local
  size_t total;
  int slot_g, slot_r;                                  // words per sender slot in ll_g / ll_r
};

EpLayout ep_layout(int world, int max_rows, int H, int k) {
  EpLayout L;
  const size_t R = (size_t)world * max_rows;
  L.slot_g = max_rows * (H / 2 + 2 * k);               // x as u32 words, ids, gates
  L.slot_r = 2 * max_rows * H;                         // routed partials, shared partials
  size_t o = 0;
  L.ll_g = o;      o += up256((size_t)world * L.slot_g * 8);
  L.ll_r = o;      o += up256((size_t)world * L.slot_r * 8);
  L.ctr = o;       o += 512;
  L.err = o;       o += 256;
  L.recv_x = o;    o += up256(R * H * 2);
  L.recv_w = o;    o += up256(R * k * 4);
  L.ids_local = o; o += up256(R * k * 4);
  L.part = o;      o += up256(R * H * 4);
  L.part_sh = o;   o += up256(R * H * 4);
  L.total = o;
  return L;
}

struct EpArgs {
  char* base[kMaxWorld];   // region of every rank, as mapped in this process (own at [rank])
  EpLayout L;
  int world, rank, rows, H, k;
  int first_expert, local_experts;
  int split;               // 1: the shared expert's partial sums travel too (second half of a slot)
  const void* x;           // [rows, H] bf16 (dispatch)
  const int32_t* ids;      // [rows, k] global ids
  const float* gates;      // [rows, k]
  void* out;               // [rows, H] bf16 (combine)
  uint64_t timeout_ns;
};

// One exchange word: 4 data bytes and the call's epoch in a single 8-byte
// store, so a reader that sees the epoch sees the data (no fence, no flag).
__device__ __forceinline__ void st_ll(uint2* p, uint32_t v, uint32_t epoch) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v), "r"(epoch) : "memory");
}

__device__ __forceinline__ uint2 ld_ll(const uint2* p) {
  uint2 r;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
  return r;
}

// Poll one word until it carries `epoch` (bounded by the communicator's
// timeout from t0, or an abort raised elsewhere); returns its data word.
__device__ __forceinline__ uint32_t wait_ll(const uint2* p, uint32_t epoch, uint64_t t0, uint64_t timeout_ns,
                                            volatile int* abort, bool& ok) {
  if (!ok) return 0u;
  for (uint32_t it = 0;; ++it) {
    const uint2 v = ld_ll(p);
    if (v.y == epoch) return v.x;
    if ((it & 255u) == 255u && (*abort || ds::ptx::globaltimer_ns() - t0 > timeout_ns)) {
      ok = false;
      return 0u;
    }
  }
}

__device__ __forceinline__ void report_timeout(int* err, volatile int* abort) {
  atomicOr(err, kErrTimeout);
  *abort = 1;
}

// This block's epoch: its own counter + 1 (every block of every rank runs
// once per call, so the counters agree across blocks and ranks).
__device__ __forceinline__ bool block_epoch(char* own, const EpLayout& L, int slot, uint32_t& epoch) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    uint32_t* ctr = reinterpret_cast<uint32_t*>(own + L.ctr) + slot;
    s_epoch = *ctr + 1;
    *ctr = s_epoch;
    s_abort = *reinterpret_cast<volatile int*>(own + L.err + 4);
  }
  __syncthreads();
  epoch = s_epoch;
  return s_abort == 0;
}

// Block (q, part): push this rank's rows (x words, global ids, gates) into
// slot `rank` of rank q's dispatch area, then take q's rows from slot q of
// our own area into the local buffers the decode kernels read (ids rewritten
// to local expert ids, -1 where another rank owns the expert).
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(const __grid_constant__ EpArgs a) {
  ds::ptx::wait_prior_grid();        // x / ids / gates come from the previous kernel (router)
  ds::ptx::launch_dependents();
  char* own = a.base[a.rank];
  int* err = reinterpret_cast<int*>(own + a.L.err);
  volatile int* abort = err + 1;
  const int q = blockIdx.x / kDispatchBlocks, part = blockIdx.x % kDispatchBlocks;
  uint32_t epoch;
  if (!block_epoch(own, a.L, blockIdx.x, epoch)) return;
  const int b = a.rows, H = a.H, k = a.k;
  const int nx = b * H / 2, n = nx + 2 * b * k;
  const uint32_t* xw = static_cast<const uint32_t*>(a.x);
  const uint32_t* iw = reinterpret_cast<const uint32_t*>(a.ids);
  const uint32_t* gw = reinterpret_cast<const uint32_t*>(a.gates);
  uint2* dst = reinterpret_cast<uint2*>(a.base[q] + a.L.ll_g) + (size_t)a.rank * a.L.slot_g;
  for (int w = part * kEpThreads + threadIdx.x; w < n; w += kDispatchBlocks * kEpThreads) {
    const uint32_t v = w < nx ? xw[w] : (w < nx + b * k ? iw[w - nx] : gw[w - nx - b * k]);
    st_ll(dst + w, v, epoch);
  }
  const uint2* src = reinterpret_cast<const uint2*>(own + a.L.ll_g) + (size_t)q * a.L.slot_g;
  uint32_t* rx = reinterpret_cast<uint32_t*>(own + a.L.recv_x) + (size_t)q * nx;
  int32_t* li = reinterpret_cast<int32_t*>(own + a.L.ids_local) + (size_t)q * b * k;
  uint32_t* rw = reinterpret_cast<uint32_t*>(own + a.L.recv_w) + (size_t)q * b * k;
  const uint64_t t0 = ds::ptx::globaltimer_ns();
  bool ok = true;
  for (int w = part * kEpThreads + threadIdx.x; w < n; w += kDispatchBlocks * kEpThreads) {
    const uint32_t v = wait_ll(src + w, epoch, t0, a.timeout_ns, abort, ok);
    if (w < nx) {
      rx[w] = v;
    } else if (w < nx + b * k) {
      const int32_t e = (int32_t)v;
      li[w - nx] = (ok && e >= a.first_expert && e < a.first_expert + a.local_experts) ? e - a.first_expert : -1;
    } else {
      rw[w - nx - b * k] = v;
    }
  }
  if (!ok) report_timeout(err, abort);
}

// Block (q, part): push the partial rows of rank q's tokens (and, split, the
// shared expert's) into slot `rank` of q's combine area; then every block
// sums its share of our b * H outputs over the G slots in rank order.
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(const __grid_constant__ EpArgs a) {
  ds::ptx::wait_prior_grid();        // partial rows come from the decode kernels
  ds::ptx::launch_dependents();
  char* own = a.base[a.rank];
  int* err = reinterpret_cast<int*>(own + a.L.err);
  volatile int* abort = err + 1;
  const int q = blockIdx.x / kCombineBlocks, part = blockIdx.x % kCombineBlocks;
  uint32_t epoch;
  if (!block_epoch(own, a.L, 64 + blockIdx.x, epoch)) return;
  const int b = a.rows, H = a.H, G = a.world;
  const int ne = b * H;
  {
    const uint32_t* pr = reinterpret_cast<const uint32_t*>(own + a.L.part) + (size_t)q * ne;
    const uint32_t* ps = reinterpret_cast<const uint32_t*>(own + a.L.part_sh) + (size_t)q * ne;
    uint2* dst = reinterpret_cast<uint2*>(a.base[q] + a.L.ll_r) + (size_t)a.rank * a.L.slot_r;
    const int n = a.split ? 2 * ne : ne;
    for (int w = part * kEpThreads + threadIdx.x; w < n; w += kCombineBlocks * kEpThreads)
      st_ll(dst + w, w < ne ? pr[w] : ps[w - ne], epoch);
  }
  const uint2* src = reinterpret_cast<const uint2*>(own + a.L.ll_r);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
  const uint64_t t0 = ds::ptx::globaltimer_ns();
  bool ok = true;
  for (int i = blockIdx.x * kEpThreads + threadIdx.x; i < ne; i += gridDim.x * kEpThreads) {
    float acc = 0.0f;
    for (int j = 0; j < G; ++j)
      acc += __uint_as_float(wait_ll(src + (size_t)j * a.L.slot_r + i, epoch, t0, a.timeout_ns, abort, ok));
    if (a.split) {
      // the shared expert's sum over the ranks, rounded to bf16 before it is
      // added, as the unsplit layer does
      float sh = 0.0f;
      for (int j = 0; j < G; ++j)
        sh += __uint_as_float(wait_ll(src + (size_t)j * a.L.slot_r + ne + i, epoch, t0, a.timeout_ns, abort, ok));
      acc += __bfloat162float(__float2bfloat16_rn(sh));
    }
    out[i] = __float2bfloat16_rn(acc);
  }
  if (!ok) report_timeout(err, abort);
}

}  // namespace

struct DsEp {
  int world, rank, max_rows, hidden, top_k, device;
  uint64_t timeout_ns;
  EpLayout L;
  char* own;                 // cudaMalloc'd region
  char* base[kMaxWorld];     // every rank's region in this process
  bool opened[kMaxWorld];    // base[j] came from cudaIpcOpenMemHandle
  bool connected;
};

extern "C" int ds_ep_create(int world, int rank, int max_rows, int hidden, int top_k, int timeout_ms,
                            DsEp** ep) {
  DS_REQUIRE(ep != nullptr, DS_EINVAL, "ep_create: null output");
  *ep = nullptr;
  DS_REQUIRE(world >= 1 && world <= kMaxWorld, DS_EINVAL, "ep_create: world %d outside 1..%d", world, kMaxWorld);
  DS_REQUIRE(rank >= 0 && rank < world, DS_EINVAL, "ep_create: rank %d outside 0..%d", rank, world - 1);
  DS_REQUIRE(max_rows >= 1 && world * max_rows <= ds::decode::kMaxTokens, DS_EINVAL,
             "ep_create: world * max_rows = %d outside 1..%d", world * max_rows, ds::decode::kMaxTokens);
  DS_REQUIRE(hidden > 0 && hidden % 8 == 0, DS_EINVAL, "ep_create: hidden must be a positive multiple of 8");
  DS_REQUIRE(top_k >= 1 && top_k <= 32, DS_EINVAL, "ep_create: top_k %d outside 1..32", top_k);
  DS_REQUIRE(timeout_ms > 0, DS_EINVAL, "ep_create: timeout_ms must be positive");
  DsEp* e = new DsEp;
  memset(e, 0, sizeof(*e));
  e->world = world;
  e->rank = rank;
  e->max_rows = max_rows;
  e->hidden = hidden;
  e->top_k = top_k;
  e->timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  e->L = ep_layout(world, max_rows, hidden, top_k);
  cudaError_t rc = cudaGetDevice(&e->device);
  if (rc == cudaSuccess) rc = cudaMalloc(reinterpret_cast<void**>(&e->own), e->L.total);
  if (rc == cudaSuccess) rc = cudaMemset(e->own, 0, e->L.total);
  if (rc == cudaSuccess) rc = cudaDeviceSynchronize();
  if (rc != cudaSuccess) {
    if (e->own) cudaFree(e->own);
    delete e;
    return ds::cuda_status(rc, "ep_create: region allocation");
  }
  e->base[rank] = e->own;
  *ep = e;
  return DS_OK;
}

extern "C" size_t ds_ep_region_bytes(int world, int max_rows, int hidden, int top_k) {
  return ep_layout(world, max_rows, hidden, top_k).total;
}

extern "C" int ds_ep_ipc_handle(DsEp* ep, void* handle) {
  DS_REQUIRE(ep != nullptr && handle != nullptr, DS_EINVAL, "ep_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  DS_CHECK_CUDA(cudaIpcGetMemHandle(&h, ep->own));
  static_assert(sizeof(h) == DS_EP_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return DS_OK;
}

extern "C" int ds_ep_connect(DsEp* ep, const void* handles) {
  DS_REQUIRE(ep != nullptr && handles != nullptr, DS_EINVAL, "ep_connect: null argument");
  DS_REQUIRE(!ep->connected, DS_EINVAL, "ep_connect: already connected");
  const char* hs = static_cast<const char*>(handles);
  for (int j = 0; j < ep->world; ++j) {
    if (j == ep->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)j * DS_EP_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const cudaError_t rc = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (rc != cudaSuccess) {
      for (int i = 0; i < j; ++i)
        if (ep->opened[i]) {
          cudaIpcCloseMemHandle(ep->base[i]);
          ep->opened[i] = false;
          ep->base[i] = nullptr;
        }
      return ds::cuda_status(rc, "ep_connect: cudaIpcOpenMemHandle");
    }
    ep->base[j] = static_cast<char*>(p);
    ep->opened[j] = true;
  }
  ep->connected = true;
  return DS_OK;
}

extern "C" int ds_ep_connect_peers(DsEp* ep, DsEp* const* all) {
  DS_REQUIRE(ep != nullptr && all != nullptr, DS_EINVAL, "ep_connect_peers: null argument");
  DS_REQUIRE(!ep->connected, DS_EINVAL, "ep_connect_peers: already connected");
  DS_REQUIRE(all[ep->rank] == ep, DS_EINVAL, "ep_connect_peers: all[rank] must be this communicator");
  for (int j = 0; j < ep->world; ++j) {
    const DsEp* o = all[j];
    DS_REQUIRE(o != nullptr && o->world == ep->world && o->rank == j && o->max_rows == ep->max_rows &&
                   o->hidden == ep->hidden && o->top_k == ep->top_k,
               DS_EINVAL, "ep_connect_peers: communicator %d does not match", j);
  }
  for (int j = 0; j < ep->world; ++j) {
    if (j == ep->rank) continue;
    if (all[j]->device != ep->device) {
      int can = 0;
      DS_CHECK_CUDA(cudaDeviceCanAccessPeer(&can, ep->device, all[j]->device));
      DS_REQUIRE(can, DS_ENOTSUP, "ep_connect_peers: device %d cannot access device %d", ep->device,
                 all[j]->device);
      const cudaError_t rc = cudaDeviceEnablePeerAccess(all[j]->device, 0);
      if (rc == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else DS_CHECK_CUDA(rc);
    }
    ep->base[j] = all[j]->own;
  }
  ep->connected = true;
  return DS_OK;
}

extern "C" int ds_ep_status(DsEp* ep, int32_t* err) {
  DS_REQUIRE(ep != nullptr && err != nullptr, DS_EINVAL, "ep_status: null argument");
  int32_t v[2] = {0, 0};
  DS_CHECK_CUDA(cudaMemcpy(v, ep->own + ep->L.err, sizeof(v), cudaMemcpyDeviceToHost));
  *err = v[0];
  return DS_OK;
}

extern "C" int ds_ep_destroy(DsEp* ep) {
  if (ep == nullptr) return DS_OK;
  cudaError_t first = cudaSuccess;
  for (int j = 0; j < ep->world; ++j)
    if (ep->opened[j]) {
      const cudaError_t rc = cudaIpcCloseMemHandle(ep->base[j]);
      if (first == cudaSuccess) first = rc;
    }
  if (ep->own) {
    const cudaError_t rc = cudaFree(ep->own);
    if (first == cudaSuccess) first = rc;
  }
  delete ep;
  if (first != cudaSuccess) return ds::cuda_status(first, "ep_destroy");
  return DS_OK;
}

extern "C" int ds_ep_decode_workspace_size(DsEp* ep, const DsMoeDesc* desc, int64_t rows, size_t* bytes) {
  DS_REQUIRE(ep != nullptr && desc != nullptr && bytes != nullptr, DS_EINVAL, "ep_decode_workspace_size: null");
  DS_REQUIRE(rows >= 1 && rows <= ep->max_rows, DS_EINVAL, "ep_decode_workspace_size: rows %lld outside 1..%d",
             (long long)rows, ep->max_rows);
  const int T = (int)(ep->world * rows);
  *bytes = desc->w1.format == DS_FMT_Q3 ? ds::decode::q3_workspace_bytes(*desc, T)
                                        : ds::decode::t5_workspace_bytes(*desc, T);
  return DS_OK;
}

extern "C" int ds_ep_decode(DsEp* ep, const DsMoeDesc* desc, int32_t first_expert, const void* x, int64_t rows,
                            const int32_t* topk_ids, const float* topk_w, void* out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  DS_REQUIRE(ep != nullptr && desc != nullptr, DS_EINVAL, "ep_decode: null handle or descriptor");
  DS_REQUIRE(ep->connected || ep->world == 1, DS_EINVAL, "ep_decode: communicator not connected");
  DS_REQUIRE(x && topk_ids && topk_w && out && workspace, DS_EINVAL, "ep_decode: null pointer");
  DS_REQUIRE(rows >= 1 && rows <= ep->max_rows, DS_EINVAL, "ep_decode: rows %lld outside 1..%d", (long long)rows,
             ep->max_rows);
  DS_REQUIRE(desc->hidden == ep->hidden && desc->top_k == ep->top_k, DS_EINVAL,
             "ep_decode: descriptor hidden/top_k differ from the communicator's");
  DS_REQUIRE(first_expert >= 0 && desc->n_experts > 0, DS_EINVAL, "ep_decode: bad expert range");
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 8) && ds::aligned(workspace, 256), DS_EALIGN,
             "ep_decode: x 16-byte, out 8-byte, workspace 256-byte aligned");
  int dev = -1;
  DS_CHECK_CUDA(cudaGetDevice(&dev));
  DS_REQUIRE(dev == ep->device, DS_EINVAL, "ep_decode: current device %d, communicator device %d", dev,
             ep->device);
  const int G = ep->world, b = (int)rows, T = G * b;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  EpArgs a;
  memset(&a, 0, sizeof(a));
  for (int j = 0; j < G; ++j) a.base[j] = ep->base[j];
  a.L = ep->L;
  a.world = G;
  a.rank = ep->rank;
  a.rows = b;
  a.H = ep->hidden;
  a.k = ep->top_k;
  a.first_expert = first_expert;
  a.local_experts = desc->n_experts;
  a.x = x;
  a.ids = topk_ids;
  a.gates = topk_w;
  a.out = out;
  a.timeout_ns = ep->timeout_ns;

  // decode over the gathered rows; the t5 path is required (f32 partial rows
  // with the shared expert restricted to this rank's rows)
  ds::decode::DecodeArgs d;
  d.d = *desc;
  d.d.out_f32 = 1;
  d.x = ep->own + ep->L.recv_x;
  d.x_f32 = 0;
  d.tokens = T;
  d.ids = reinterpret_cast<const int32_t*>(ep->own + ep->L.ids_local);
  d.gates = reinterpret_cast<const float*>(ep->own + ep->L.recv_w);
  d.out = ep->own + ep->L.part;
  d.h = nullptr;
  d.max_slots = std::min(T * desc->top_k, desc->n_experts);
  d.h_stride = 0;
  d.err = static_cast<int*>(workspace);
  d.sh_row0 = ep->rank * b;
  d.sh_row1 = ep->rank * b + b;
  // shared expert: when its inter splits into G slices of 256, rank r
  // evaluates slice r for all gathered rows (f32 partial sums, summed over
  // the ranks in the combine); otherwise each rank evaluates all of it for
  // its own rows
  const bool sh = desc->shared_w1 != nullptr;
  a.split = sh && desc->shared_inter % (256 * G) == 0;     // slices of 256 suit both decode paths
  if (a.split) {
    const int Is = desc->shared_inter, Isl = Is / G, r = ep->rank;
    d.d.shared_inter = Isl;
    d.d.shared_w1 = static_cast<const __nv_bfloat16*>(desc->shared_w1) + (size_t)r * Isl * desc->hidden;
    d.d.shared_w3 = static_cast<const __nv_bfloat16*>(desc->shared_w3) + (size_t)r * Isl * desc->hidden;
    d.d.shared_w2 = static_cast<const __nv_bfloat16*>(desc->shared_w2) + (size_t)r * Isl;
    d.sh_w2_ld = Is;
    d.out_sh = reinterpret_cast<float*>(ep->own + ep->L.part_sh);
  }
  const bool t5 = ds::decode::t5_supported(d);
  const bool q3 = !t5 && ds::decode::q3_supported(d);
  DS_REQUIRE(t5 || q3, DS_ENOTSUP,
             "ep_decode: needs FP4 banks with scale atoms (hidden and inter multiples of 1024) or Q3 banks "
             "(multiples of 128)");

  // programmatic dependent launches: each kernel starts while its
  // predecessor drains and waits for it (griddepcontrol.wait) before it
  // reads what the predecessor wrote
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(kEpThreads);
  cfg.gridDim = dim3(G * kDispatchBlocks);
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, ep_dispatch_kernel, a));
  int rc = t5 ? ds::decode::launch_t5(d, workspace, workspace_bytes, st)
              : ds::decode::launch_q3(d, workspace, workspace_bytes, st);
  if (rc != DS_OK) return rc;
  cfg.gridDim = dim3(G * kCombineBlocks);
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, ep_combine_kernel, a));
  return DS_OK;
}
