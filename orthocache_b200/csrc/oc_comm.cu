// Sequence-parallel exchange over NCCL, behind the C ABI: a host that is not
// Python drives the sharded path through these entry points with an NCCL
// communicator (one rank per GPU).
//
//   oc_exchange_stratified   build_stratified (benchmarks/phase_e_stratified.py:
//                            164-273): count all-gather, capacity bucket from
//                            the largest count, every rank's first `bucket`
//                            retained K/V blocks all-gathered, valid-slot index
//   oc_alltoallv_heads       a true AllToAllv (alltoallv.py:217-259 moves every
//                            retained block to every rank; here each rank
//                            receives only the KV heads it owns, with per-peer
//                            sizes from the count all-gather): grouped
//                            ncclSend / ncclRecv
//   oc_decode_step_sharded   one sequence-parallel decode layer: the fused
//                            layer's (m, l, o) partial of this shard, an
//                            all-gather of the packed partials, the
//                            log-sum-exp merge (distributed_attention.py:95-128
//                            applied across shards)
//
// NCCL is resolved at run time, not linked: the copy already loaded in the
// process (the one that created the caller's communicator, e.g. PyTorch's) if
// there is one, else libnccl.so.2 (or the path in OC_NCCL_LIBRARY).  Only the
// types come from nccl.h; the ABI of these calls is stable across NCCL 2.x.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "oc_common.cuh"

namespace oc {
namespace {

struct NcclApi {
  int version = 0;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;
bool g_nccl_tried = false;

template <typename F>
bool sym(void* h, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(h, name));
  return f != nullptr;
}

// The process's NCCL, loaded once.
const NcclApi* nccl() {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (g_nccl_tried) return g_nccl.version ? &g_nccl : nullptr;
  g_nccl_tried = true;
  void* h = nullptr;
  if (const char* p = getenv("OC_NCCL_LIBRARY")) h = dlopen(p, RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) return nullptr;
  NcclApi a;
  bool ok = sym(h, "ncclGetVersion", a.GetVersion) && sym(h, "ncclGetUniqueId", a.GetUniqueId) &&
            sym(h, "ncclCommInitRank", a.CommInitRank) && sym(h, "ncclCommDestroy", a.CommDestroy) &&
            sym(h, "ncclCommAbort", a.CommAbort) && sym(h, "ncclCommCount", a.CommCount) &&
            sym(h, "ncclCommUserRank", a.CommUserRank) && sym(h, "ncclCommGetAsyncError", a.CommGetAsyncError) &&
            sym(h, "ncclAllGather", a.AllGather) && sym(h, "ncclSend", a.Send) && sym(h, "ncclRecv", a.Recv) &&
            sym(h, "ncclGroupStart", a.GroupStart) && sym(h, "ncclGroupEnd", a.GroupEnd) &&
            sym(h, "ncclGetErrorString", a.GetErrorString);
  if (!ok || a.GetVersion(&a.version) != ncclSuccess) return nullptr;
  g_nccl = a;
  return &g_nccl;
}

int nccl_err(const NcclApi* n, ncclResult_t r, const char* what) {
  return set_error(OC_ERR_COMM, "%s: NCCL error %d (%s)", what, (int)r, n->GetErrorString(r));
}

#define OC_NCCL(call, what)                          \
  do {                                               \
    ncclResult_t r_ = (call);                        \
    if (r_ != ncclSuccess) return nccl_err(n, r_, what); \
  } while (0)

int comm_shape(const NcclApi* n, ncclComm_t c, int* nranks, int* rank, const char* what) {
  OC_NCCL(n->CommCount(c, nranks), what);
  OC_NCCL(n->CommUserRank(c, rank), what);
  return OC_OK;
}

int esize(int dtype) { return dtype == OC_BF16 ? 2 : 4; }
ncclDataType_t ntype(int dtype) { return dtype == OC_BF16 ? ncclBfloat16 : ncclFloat32; }

// Every rank's count (one int32 each) on the device and on the host.
int gather_counts(const NcclApi* n, ncclComm_t c, const int32_t* count, int32_t* all_counts, int nranks,
                  std::vector<int>& host, cudaStream_t st, const char* what) {
  OC_NCCL(n->AllGather(count, all_counts, 1, ncclInt32, c, st), what);
  host.assign(nranks, 0);
  cudaError_t e = cudaMemcpyAsync(host.data(), all_counts, sizeof(int) * nranks, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: count copy: %s", what, cudaGetErrorString(e));
  return OC_OK;
}

// send[p][i][t][hl][d] = src[idx[i] * bs + t][p * hper + hl][d] for i < count:
// the retained blocks of this shard, split by the KV heads each rank owns.
// One 16-byte vector per thread.
__global__ void pack_heads_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ idx,
                                  const int32_t* __restrict__ count, int P, int hper, int bs, int vec_per_head,
                                  int H, uint4* __restrict__ dst) {
  const int n = *count;
  const int64_t per_peer = (int64_t)n * bs * hper * vec_per_head;
  const int64_t total = per_peer * P;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e;
    const int c = (int)(r % vec_per_head); r /= vec_per_head;
    const int hl = (int)(r % hper); r /= hper;
    const int t = (int)(r % bs); r /= bs;
    const int i = (int)(r % n);
    const int p = (int)(r / n);
    const int64_t tok = (int64_t)idx[i] * bs + t;
    dst[e] = src[(tok * H + (int64_t)p * hper + hl) * vec_per_head + c];
  }
}

}  // namespace
}  // namespace oc

using namespace oc;

extern "C" int oc_nccl_version(void) {
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  return n->version;
}

extern "C" int oc_comm_unique_id(void* id_out) {
  OC_REQUIRE(id_out, OC_ERR_NULL, "oc_comm_unique_id: id_out is NULL");
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  OC_NCCL(n->GetUniqueId(reinterpret_cast<ncclUniqueId*>(id_out)), "oc_comm_unique_id");
  return OC_OK;
}

extern "C" int oc_comm_init(void** comm_out, const void* id, int nranks, int rank) {
  OC_REQUIRE(comm_out && id, OC_ERR_NULL, "oc_comm_init: NULL argument");
  OC_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, OC_ERR_SHAPE, "oc_comm_init: rank %d of %d", rank, nranks);
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  OC_NCCL(n->CommInitRank(&c, nranks, uid, rank), "oc_comm_init");
  *comm_out = c;
  return OC_OK;
}

extern "C" int oc_comm_destroy(void* comm) {
  if (!comm) return OC_OK;
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  OC_NCCL(n->CommDestroy(reinterpret_cast<ncclComm_t>(comm)), "oc_comm_destroy");
  return OC_OK;
}

extern "C" int oc_comm_check(void* comm) {
  OC_REQUIRE(comm, OC_ERR_NULL, "oc_comm_check: comm is NULL");
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  ncclResult_t async = ncclSuccess;
  OC_NCCL(n->CommGetAsyncError(reinterpret_cast<ncclComm_t>(comm), &async), "oc_comm_check");
  if (async == ncclInProgress) return OC_OK;
  if (async != ncclSuccess) return nccl_err(n, async, "oc_comm_check: asynchronous error");
  return OC_OK;
}

extern "C" int oc_comm_abort(void* comm) {
  if (!comm) return OC_OK;
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  OC_NCCL(n->CommAbort(reinterpret_cast<ncclComm_t>(comm)), "oc_comm_abort");
  return OC_OK;
}

extern "C" size_t oc_exchange_workspace_bytes(int num_blocks, int kv_heads, int head_dim, int dtype,
                                              int block_size) {
  if (num_blocks < 0 || kv_heads < 1 || head_dim < 1 || block_size < 1 || (dtype != OC_F32 && dtype != OC_BF16))
    return 0;
  const size_t tensor = (size_t)num_blocks * block_size * kv_heads * head_dim * esize(dtype);
  return 2 * ((tensor + 255) / 256 * 256);
}

namespace {
int exchange_args(const void* comm, const void* k, const void* v, int dtype, const int32_t* idx,
                  const int32_t* count, int nb, int H, int D, int bs, const void* k_recv, const void* v_recv,
                  const int32_t* all_counts, void* ws, size_t ws_bytes, const char* what) {
  OC_REQUIRE(comm && k && v && idx && count && k_recv && v_recv && all_counts && ws, OC_ERR_NULL, "%s: NULL argument",
             what);
  OC_REQUIRE(dtype == OC_F32 || dtype == OC_BF16, OC_ERR_DTYPE, "%s: dtype %d", what, dtype);
  OC_REQUIRE(nb >= 1 && H >= 1 && D >= 1 && bs >= 1, OC_ERR_SHAPE, "%s: bad shape", what);
  OC_REQUIRE(aligned16(k) && aligned16(v) && aligned16(k_recv) && aligned16(v_recv) && aligned16(ws), OC_ERR_ALIGN,
             "%s: buffers must be 16-byte aligned", what);
  const size_t need = oc_exchange_workspace_bytes(nb, H, D, dtype, bs);
  OC_REQUIRE(ws_bytes >= need, OC_ERR_CAPACITY, "%s: workspace %zu < %zu bytes", what, ws_bytes, need);
  return OC_OK;
}
}  // namespace

extern "C" int oc_exchange_stratified(void* comm, const void* k, const void* v, int dtype, const int32_t* idx,
                                      const int32_t* count, int num_blocks, int kv_heads, int head_dim,
                                      int block_size, void* k_recv, void* v_recv, int32_t* all_counts,
                                      int32_t* order, int32_t* total, int* bucket_out, void* workspace,
                                      size_t workspace_bytes, oc_stream_t stream) {
  const char* what = "oc_exchange_stratified";
  int rc = exchange_args(comm, k, v, dtype, idx, count, num_blocks, kv_heads, head_dim, block_size, k_recv, v_recv,
                         all_counts, workspace, workspace_bytes, what);
  if (rc) return rc;
  OC_REQUIRE(order && total, OC_ERR_NULL, "%s: order / total is NULL", what);
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  ncclComm_t c = reinterpret_cast<ncclComm_t>(comm);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int P = 0, me = 0;
  if ((rc = comm_shape(n, c, &P, &me, what))) return rc;
  std::vector<int> h;
  if ((rc = gather_counts(n, c, count, all_counts, P, h, st, what))) return rc;
  const int gmax = *std::max_element(h.begin(), h.end());
  // the bucket sizes the collective, so it is known on the host: the one
  // synchronisation of the exchange (the reference's pmax + lax.switch)
  const int bucket = oc_stratified_bucket(num_blocks, gmax);
  const int64_t block_elems = (int64_t)block_size * kv_heads * head_dim;
  const size_t tensor = (size_t)num_blocks * block_elems * esize(dtype);
  char* sk = static_cast<char*>(workspace);
  char* sv = sk + (tensor + 255) / 256 * 256;
  if ((rc = oc_gather_blocks(k, dtype, 1, num_blocks, block_elems, idx, num_blocks, count, sk, bucket, 1, stream)))
    return rc;
  if ((rc = oc_gather_blocks(v, dtype, 1, num_blocks, block_elems, idx, num_blocks, count, sv, bucket, 1, stream)))
    return rc;
  const size_t elems = (size_t)bucket * block_elems;
  OC_NCCL(n->GroupStart(), what);
  OC_NCCL(n->AllGather(sk, k_recv, elems, ntype(dtype), c, st), what);
  OC_NCCL(n->AllGather(sv, v_recv, elems, ntype(dtype), c, st), what);
  OC_NCCL(n->GroupEnd(), what);
  if ((rc = oc_exchange_index(all_counts, P, bucket, order, total, nullptr, stream))) return rc;
  if (bucket_out) *bucket_out = bucket;
  return OC_OK;
}

extern "C" int oc_alltoallv_heads(void* comm, const void* k, const void* v, int dtype, const int32_t* idx,
                                  const int32_t* count, int num_blocks, int kv_heads, int head_dim, int block_size,
                                  void* k_recv, void* v_recv, int32_t* all_counts, int* total_out, void* workspace,
                                  size_t workspace_bytes, oc_stream_t stream) {
  const char* what = "oc_alltoallv_heads";
  int rc = exchange_args(comm, k, v, dtype, idx, count, num_blocks, kv_heads, head_dim, block_size, k_recv, v_recv,
                         all_counts, workspace, workspace_bytes, what);
  if (rc) return rc;
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  ncclComm_t c = reinterpret_cast<ncclComm_t>(comm);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int P = 0, me = 0;
  if ((rc = comm_shape(n, c, &P, &me, what))) return rc;
  OC_REQUIRE(kv_heads % P == 0, OC_ERR_SHAPE, "%s: kv_heads %d is not a multiple of the %d ranks", what, kv_heads, P);
  OC_REQUIRE((head_dim * esize(dtype)) % 16 == 0, OC_ERR_SHAPE, "%s: a head row must be whole 16-byte vectors", what);
  std::vector<int> h;
  if ((rc = gather_counts(n, c, count, all_counts, P, h, st, what))) return rc;
  const int hper = kv_heads / P;
  const int vph = head_dim * esize(dtype) / 16;
  const int mine = h[me];
  const size_t blk = (size_t)block_size * hper * head_dim * esize(dtype);  // one block of one rank's heads
  const size_t tensor = (size_t)num_blocks * block_size * kv_heads * head_dim * esize(dtype);
  char* sk = static_cast<char*>(workspace);
  char* sv = sk + (tensor + 255) / 256 * 256;
  if (mine > 0) {
    const int64_t vecs = (int64_t)mine * block_size * hper * vph * P;
    const int grid = (int)std::min<int64_t>((vecs + 255) / 256, 148 * 16);
    pack_heads_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(k), idx, count, P, hper, block_size, vph,
                                            kv_heads, reinterpret_cast<uint4*>(sk));
    pack_heads_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(v), idx, count, P, hper, block_size, vph,
                                            kv_heads, reinterpret_cast<uint4*>(sv));
    if ((rc = check_launch("pack_heads_kernel"))) return rc;
  }
  // peer p gets my blocks of its heads; I get peer p's blocks of my heads,
  // placed after those of the lower ranks (rank order, as the reference's
  // unpack_received_blocks leaves them)
  OC_NCCL(n->GroupStart(), what);
  size_t off = 0;
  for (int p = 0; p < P; ++p) {
    const size_t send_elems = (size_t)mine * blk / esize(dtype), recv_elems = (size_t)h[p] * blk / esize(dtype);
    if (send_elems) {
      OC_NCCL(n->Send(sk + (size_t)p * mine * blk, send_elems, ntype(dtype), p, c, st), what);
      OC_NCCL(n->Send(sv + (size_t)p * mine * blk, send_elems, ntype(dtype), p, c, st), what);
    }
    if (recv_elems) {
      OC_NCCL(n->Recv(static_cast<char*>(k_recv) + off * blk, recv_elems, ntype(dtype), p, c, st), what);
      OC_NCCL(n->Recv(static_cast<char*>(v_recv) + off * blk, recv_elems, ntype(dtype), p, c, st), what);
    }
    off += h[p];
  }
  OC_NCCL(n->GroupEnd(), what);
  if (total_out) *total_out = (int)off;
  return OC_OK;
}

namespace oc {
namespace {

// Layout of the sharded decode workspace: the decode step's workspace, the
// packed send partial and P received partials of the NCCL path, the table of
// the P ranks' exchange-region addresses, then this rank's exchange region.
struct ShardedLayout {
  size_t base, part, table, region, bytes;
  int NG;
};

ShardedLayout sharded_layout(int P, int B, int Sq, int Hq, int Hkv, int D, int S) {
  ShardedLayout L = {};
  L.base = oc_decode_step_workspace_bytes(B, Sq, Hq, Hkv, D, S);
  if (!L.base || P < 1) return L;
  const size_t rows = (size_t)B * Sq * Hq;
  L.part = (rows * (D + 2) * sizeof(float) + 255) / 256 * 256;
  L.NG = B * Hkv;
  L.table = L.base + L.part * (1 + P);
  L.region = L.table + ((size_t)P * sizeof(void*) + 255) / 256 * 256;
  L.bytes = L.region + xchg_region_bytes(P, L.NG);
  return L;
}

// Workspaces whose exchange regions are mapped into every rank (host side).
struct Connection {
  int P, rank;
  std::vector<void*> opened;  // peer allocations mapped by cudaIpcOpenMemHandle
};
std::mutex g_conn_mu;
std::vector<std::pair<void*, Connection>> g_conns;

Connection* find_conn(void* ws) {
  for (auto& c : g_conns)
    if (c.first == ws) return &c.second;
  return nullptr;
}

using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  }
  return fn;
}

struct IpcRecord {
  cudaIpcMemHandle_t handle;
  uint64_t offset;  // of the exchange region from the allocation's base
  uint64_t pad;
};

}  // namespace
}  // namespace oc

extern "C" size_t oc_decode_step_sharded_workspace_bytes(int nranks, int batch, int q_len, int q_heads,
                                                         int kv_heads, int head_dim, int seq_len) {
  return oc::sharded_layout(nranks, batch, q_len, q_heads, kv_heads, head_dim, seq_len).bytes;
}

extern "C" int oc_sharded_connect(void* comm, void* workspace, size_t workspace_bytes, int batch, int q_len,
                                  int q_heads, int kv_heads, int head_dim, int seq_len, oc_stream_t stream) {
  const char* what = "oc_sharded_connect";
  OC_REQUIRE(comm && workspace, OC_ERR_NULL, "%s: NULL argument", what);
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  ncclComm_t c = reinterpret_cast<ncclComm_t>(comm);
  int P = 0, me = 0, rc;
  if ((rc = comm_shape(n, c, &P, &me, what))) return rc;
  const ShardedLayout L = sharded_layout(P, batch, q_len, q_heads, kv_heads, head_dim, seq_len);
  OC_REQUIRE(L.bytes && workspace_bytes >= L.bytes, OC_ERR_CAPACITY, "%s: workspace %zu < %zu bytes", what,
             workspace_bytes, L.bytes);
  OC_REQUIRE(head_dim == 128 && q_len * (q_heads / kv_heads) <= 8, OC_ERR_UNSUPPORTED,
             "%s: the peer exchange serves the fused decode layer (head_dim 128, <= 8 query rows per KV head)",
             what);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  char* region = ws + L.region;
  AddrRangeFn range = addr_range_fn();
  if (!range) return set_error(OC_ERR_CUDA, "%s: cuMemGetAddressRange is unavailable", what);
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(region)) != CUDA_SUCCESS)
    return set_error(OC_ERR_CUDA, "%s: cuMemGetAddressRange failed", what);
  IpcRecord mine = {};
  cudaError_t e = cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: cudaIpcGetMemHandle: %s", what, cudaGetErrorString(e));
  mine.offset = reinterpret_cast<uint64_t>(region) - base;
  // all-gather the records through NCCL, staged in the NCCL path's receive
  // buffers (scratch at this point)
  char* stage = ws + L.base;
  const size_t rec = sizeof(IpcRecord);
  OC_REQUIRE(rec * (1 + P) <= L.part * (1 + P), OC_ERR_CAPACITY, "%s: staging too small", what);
  e = cudaMemcpyAsync(stage, &mine, rec, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  OC_NCCL(n->AllGather(stage, stage + rec, rec, ncclUint8, c, st), what);
  std::vector<IpcRecord> all(P);
  e = cudaMemcpyAsync(all.data(), stage + rec, rec * P, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  Connection conn;
  conn.P = P;
  conn.rank = me;
  std::vector<char*> table(P);
  cudaError_t open_err = cudaSuccess;
  for (int p = 0; p < P && open_err == cudaSuccess; ++p) {
    if (p == me) {
      table[p] = region;
      continue;
    }
    void* mapped = nullptr;
    open_err = cudaIpcOpenMemHandle(&mapped, all[p].handle, cudaIpcMemLazyEnablePeerAccess);
    if (open_err == cudaSuccess) {
      conn.opened.push_back(mapped);
      table[p] = static_cast<char*>(mapped) + all[p].offset;
    }
  }
  // the table, and exchange words that start at zero (call numbers start at 1)
  e = open_err;
  if (e == cudaSuccess) e = cudaMemcpyAsync(ws + L.table, table.data(), sizeof(char*) * P, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(region, 0, xchg_region_bytes(P, L.NG), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  // Agree on the outcome: every rank learns whether every other rank is
  // connected (and has its flags at zero) before any exchange, so that no
  // rank takes the peer path while another takes NCCL.
  mine.pad = e == cudaSuccess ? 0 : 1;
  cudaError_t e2 = cudaMemcpyAsync(stage, &mine, rec, cudaMemcpyHostToDevice, st);
  if (e2 != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e2));
  OC_NCCL(n->AllGather(stage, stage + rec, rec, ncclUint8, c, st), what);
  e2 = cudaMemcpyAsync(all.data(), stage + rec, rec * P, cudaMemcpyDeviceToHost, st);
  if (e2 == cudaSuccess) e2 = cudaStreamSynchronize(st);
  if (e2 != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e2));
  bool all_ok = true;
  for (int p = 0; p < P; ++p) all_ok = all_ok && all[p].pad == 0;
  if (!all_ok) {
    for (void* m : conn.opened) cudaIpcCloseMemHandle(m);
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return set_error(OC_ERR_UNSUPPORTED, "%s: another rank could not map the exchange regions", what);
  }
  std::lock_guard<std::mutex> lock(g_conn_mu);
  if (Connection* old = find_conn(workspace)) {
    for (void* m : old->opened) cudaIpcCloseMemHandle(m);
    *old = conn;
  } else {
    g_conns.emplace_back(workspace, conn);
  }
  return OC_OK;
}

extern "C" int oc_sharded_disconnect(void* workspace) {
  std::lock_guard<std::mutex> lock(g_conn_mu);
  for (size_t i = 0; i < g_conns.size(); ++i)
    if (g_conns[i].first == workspace) {
      for (void* m : g_conns[i].second.opened) cudaIpcCloseMemHandle(m);
      g_conns.erase(g_conns.begin() + i);
      return OC_OK;
    }
  return OC_OK;
}

extern "C" int oc_decode_step_sharded(void* comm, const void* q, const void* k, const void* v, int dtype, int batch,
                                      int q_len, int q_heads, int kv_heads, int head_dim, int seq_len, float tau,
                                      float zeta_max, uint8_t* keep, int32_t* perm, int32_t* count, void* out,
                                      int out_dtype, void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  const char* what = "oc_decode_step_sharded";
  OC_REQUIRE(comm && workspace && out, OC_ERR_NULL, "%s: NULL argument", what);
  const NcclApi* n = nccl();
  if (!n) return set_error(OC_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  ncclComm_t c = reinterpret_cast<ncclComm_t>(comm);
  int P = 0, me = 0, rc;
  if ((rc = comm_shape(n, c, &P, &me, what))) return rc;
  const ShardedLayout L = sharded_layout(P, batch, q_len, q_heads, kv_heads, head_dim, seq_len);
  OC_REQUIRE(L.bytes && workspace_bytes >= L.bytes, OC_ERR_CAPACITY, "%s: workspace %zu < %zu bytes", what,
             workspace_bytes, L.bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  bool connected = false;
  {
    std::lock_guard<std::mutex> lock(g_conn_mu);
    const Connection* cn = find_conn(workspace);
    connected = cn && cn->P == P && cn->rank == me;
  }
  if (connected && dtype == OC_BF16) {
    // one kernel: the fused layer merges its shard's partial with every
    // rank's through the mapped exchange regions
    PeerXchg px;
    px.bases = reinterpret_cast<char* const*>(ws + L.table);
    px.P = P;
    px.rank = me;
    rc = decode_fused(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max, keep, perm, count,
                      out, out_dtype, nullptr, nullptr, nullptr, workspace, L.base, st, &px);
    if (rc != OC_ERR_UNSUPPORTED) return rc;
  }
  const int rows = batch * q_len * q_heads;
  float* send = reinterpret_cast<float*>(ws + L.base);
  float* recv = reinterpret_cast<float*>(ws + L.base + L.part);
  // this shard's partial, packed [m (rows) | l (rows) | o (rows, D)]
  rc = oc_decode_step_partial(q, k, v, dtype, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max, keep,
                              perm, count, send, send + rows, send + 2 * (size_t)rows, workspace, L.base, stream);
  if (rc) return rc;
  // the P partials land back to back in recv, the layout the merge reads
  const size_t floats = (size_t)rows * (head_dim + 2);
  OC_NCCL(n->AllGather(send, recv, floats, ncclFloat32, c, st), what);
  return oc_merge_partials_packed(recv, P, rows, head_dim, out, out_dtype, stream);
}
