// dp_comm.cu -- the data-parallel communicator of the fused lowrank backward.
//
// Each rank (one process per GPU on one node) allocates, once, a landing buffer
// [2 parities][world sources][cap floats] and a flag array [world sources][kMaxDpCtas]
// of 64-bit call numbers in its own device memory, exports CUDA IPC handles of both,
// and opens every peer's handles.  In the backward kernel (lowrank_bwd_tm.cu) CTA i
// of every rank owns the same slice of the dU / dstatic_w buffer: it writes this
// rank's sum of its slice straight into slot [parity][rank] of every rank's landing
// buffer over NVLink (plain stores to peer memory), then stores the call number in
// flag [rank][i] of every rank, waits (bounded) until flag [src][i] of its own array
// shows the call for every source, and sums the world slots of its slice in rank
// order -- so all ranks hold the same, deterministic result, and the all-reduce
// replaces the NCCL collective that followed the kernel.  Each flag has one writer,
// so no CTA waits on another CTA's slice and no flag is contended.  Only plain
// stores and loads touch peer memory (no TMA, no switch-side reduction).
//
// The flags hold call numbers, and the call count lives on the device (advanced by
// the kernel), so calls may differ in size and the kernels can be captured in a
// CUDA graph and replayed.
// Landing slots alternate by call parity: a rank can only be two calls ahead of a
// peer once that peer has finished reading the older call's slot (a call's
// kernel waits for every peer's contribution to that call).
#include <cuda_runtime.h>

#include <string.h>

#include "../../include/dynconv.h"
#include "lowrank_tc.cuh"

namespace dynconv {

struct Comm {
  int world = 0, rank = 0, device = -1;
  int64_t cap = 0;             // floats per (parity, source) slot
  float* land = nullptr;       // own landing buffer
  unsigned long long* flags = nullptr;  // own flags [world][kMaxDpCtas]
  unsigned long long* epoch = nullptr;  // own count of completed calls
  bool connected = false;
  float* peer_land[lrtc::kMaxWorld] = {};
  unsigned long long* peer_flags[lrtc::kMaxWorld] = {};
};

namespace {

// One rank's exported blob: the two IPC handles, the device UUID (to refuse two
// ranks on one GPU, whose kernels would wait on each other), the rank and sizes.
struct Blob {
  cudaIpcMemHandle_t land, flags;
  cudaUUID_t uuid;
  int32_t rank, world;
  int64_t cap;
};

}  // namespace

bool comm_peers(const void* comm, lrtc::DpPeers* out) {
  const Comm* c = static_cast<const Comm*>(comm);
  if (!c || !c->connected) return false;
  memset(out, 0, sizeof(*out));
  out->world = c->world;
  out->rank = c->rank;
  out->cap = c->cap;
  for (int p = 0; p < c->world; ++p) {
    out->land[p] = c->peer_land[p];
    out->flags[p] = c->peer_flags[p];
  }
  out->epoch = c->epoch;
  return true;
}

int comm_device(const void* comm) { return comm ? static_cast<const Comm*>(comm)->device : -1; }

}  // namespace dynconv

using dynconv::Comm;

extern "C" {

size_t dynconv_comm_blob_bytes(void) { return sizeof(dynconv::Blob); }

int dynconv_comm_create(int world, int rank, int64_t max_floats, void** comm, void* blob) {
  using namespace dynconv;
  if (!comm || !blob) return set_error(DYNCONV_ERR_ARGUMENT, "comm_create: null pointer");
  *comm = nullptr;
  if (world < 2 || world > lrtc::kMaxWorld || rank < 0 || rank >= world)
    return set_error(DYNCONV_ERR_SHAPE, "comm_create: world %d / rank %d (world 2..%d)", world, rank, lrtc::kMaxWorld);
  if (max_floats <= 0 || max_floats % 4 != 0)
    return set_error(DYNCONV_ERR_SHAPE, "comm_create: max_floats %lld must be a positive multiple of 4",
                     (long long)max_floats);
  Comm* c = new Comm();
  c->world = world;
  c->rank = rank;
  c->cap = max_floats;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->land, (size_t)2 * world * max_floats * sizeof(float));
  const size_t nflags = (size_t)world * lrtc::kMaxDpCtas + 1;  // + the call counter
  if (e == cudaSuccess) e = cudaMalloc(&c->flags, nflags * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(c->flags, 0, nflags * sizeof(unsigned long long));
  if (e == cudaSuccess) c->epoch = c->flags + (size_t)world * lrtc::kMaxDpCtas;
  Blob b;
  memset(&b, 0, sizeof(b));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&b.land, c->land);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&b.flags, c->flags);
  cudaDeviceProp prop;
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, c->device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // the zeroed counters are in place before any peer maps them
  if (e != cudaSuccess) {
    const int s = cuda_status(e, "comm_create");
    if (c->land) cudaFree(c->land);
    if (c->flags) cudaFree(c->flags);
    delete c;
    return s;
  }
  b.uuid = prop.uuid;
  b.rank = rank;
  b.world = world;
  b.cap = max_floats;
  memcpy(blob, &b, sizeof(b));
  *comm = c;
  return DYNCONV_OK;
}

int dynconv_comm_connect(void* comm, const void* blobs) {
  using namespace dynconv;
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !blobs) return set_error(DYNCONV_ERR_ARGUMENT, "comm_connect: null pointer");
  if (c->connected) return set_error(DYNCONV_ERR_ARGUMENT, "comm_connect: already connected");
  const Blob* all = static_cast<const Blob*>(blobs);
  for (int p = 0; p < c->world; ++p) {
    if (all[p].rank != p || all[p].world != c->world || all[p].cap != c->cap)
      return set_error(DYNCONV_ERR_ARGUMENT, "comm_connect: blob %d is rank %d of %d (cap %lld), expected rank %d of %d",
                       p, all[p].rank, all[p].world, (long long)all[p].cap, p, c->world);
    for (int q = 0; q < p; ++q)
      if (memcmp(&all[p].uuid, &all[q].uuid, sizeof(cudaUUID_t)) == 0)
        return set_error(DYNCONV_ERR_UNSUPPORTED, "comm_connect: ranks %d and %d share one GPU", q, p);
  }
  int opened = 0;
  cudaError_t e = cudaSuccess;
  for (int p = 0; p < c->world && e == cudaSuccess; ++p) {
    if (p == c->rank) {
      c->peer_land[p] = c->land;
      c->peer_flags[p] = c->flags;
      continue;
    }
    void* l = nullptr;
    void* f = nullptr;
    e = cudaIpcOpenMemHandle(&l, all[p].land, cudaIpcMemLazyEnablePeerAccess);
    if (e == cudaSuccess) {
      e = cudaIpcOpenMemHandle(&f, all[p].flags, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) cudaIpcCloseMemHandle(l);
    }
    if (e == cudaSuccess) {
      c->peer_land[p] = static_cast<float*>(l);
      c->peer_flags[p] = static_cast<unsigned long long*>(f);
      ++opened;
    }
  }
  if (e != cudaSuccess) {
    for (int p = 0; p < c->world; ++p)
      if (p != c->rank && c->peer_land[p]) {
        cudaIpcCloseMemHandle(c->peer_land[p]);
        cudaIpcCloseMemHandle(c->peer_flags[p]);
        c->peer_land[p] = nullptr;
        c->peer_flags[p] = nullptr;
      }
    return cuda_status(e, "comm_connect: cudaIpcOpenMemHandle");
  }
  c->connected = true;
  return DYNCONV_OK;
}

int dynconv_comm_destroy(void* comm) {
  using namespace dynconv;
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return DYNCONV_OK;
  cudaError_t first = cudaSuccess;
  for (int p = 0; p < c->world; ++p)
    if (p != c->rank && c->peer_land[p]) {
      cudaError_t e1 = cudaIpcCloseMemHandle(c->peer_land[p]);
      cudaError_t e2 = cudaIpcCloseMemHandle(c->peer_flags[p]);
      if (first == cudaSuccess) first = e1 != cudaSuccess ? e1 : e2;
    }
  if (c->land) cudaFree(c->land);
  if (c->flags) cudaFree(c->flags);
  delete c;
  return first == cudaSuccess ? DYNCONV_OK : cuda_status(first, "comm_destroy");
}

}  // extern "C"
