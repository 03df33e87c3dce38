// Tensor parallelism over NVLink: an NCCL communicator behind the C ABI and
// the small kernels around the per-layer allreduces of the tensor-parallel
// decode (column-parallel QKV / gate_up / lm_head, row-parallel o / down).
//
// The reference has no inference-time parallelism (its only collective is a
// training all_reduce, axiomlm/train.py:296); this is the B200 build's own
// multi-GPU mode.  NCCL is resolved at run time by its soname, so the library
// shares the one the process already loaded (torch's).
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "axb_common.cuh"
#include "tp.cuh"

namespace axb {

namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
    api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
    api.comm_abort = (decltype(api.comm_abort))dlsym(h, "ncclCommAbort");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort && api.all_reduce;
  });
  return api;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return AXB_OK;
  const char* msg = nccl().error_string ? nccl().error_string(r) : "";
  set_error("%s: NCCL error %d (%s)", what, (int)r, msg);
  return AXB_ECUDA;
}
}  // namespace

int tp_allreduce(void* comm, void* buf, size_t count, int op, cudaStream_t st) {
  NcclApi& api = nccl();
  AXB_CHECK_ARG(api.ok, "tp: NCCL (libnccl.so.2) is not available");
  AXB_CHECK_ARG(comm && buf, "tp_allreduce: null communicator or buffer");
  ncclDataType_t dt;
  ncclRedOp_t ro;
  switch (op) {
    case AXB_TP_SUM_F32: dt = ncclFloat32; ro = ncclSum; break;
    case AXB_TP_SUM_F16: dt = ncclFloat16; ro = ncclSum; break;
    case AXB_TP_MAX_U64: dt = ncclUint64; ro = ncclMax; break;
    default: set_error("tp_allreduce: unknown op %d", op); return AXB_EINVAL;
  }
  return nccl_status(api.all_reduce(buf, buf, count, dt, ro, (ncclComm_t)comm, st), "tp allreduce");
}

// x[i] = fp16(x[i] + fp16(part[i])): the residual add after a row-parallel
// projection's partial sums met (transformer.py:1176-1191 rounding points)
__global__ void tp_residual_kernel(__half* __restrict__ x, const float* __restrict__ part, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    x[i] = __float2half_rn(__fadd_rn(__half2float(x[i]), __half2float(__float2half_rn(part[i]))));
}

int tp_residual(__half* x, const float* part, int n, cudaStream_t st) {
  tp_residual_kernel<<<std::min((n + 255) / 256, 4 * num_sms()), 256, 0, st>>>(x, part, n);
  return launch_status("tp residual");
}

// argmax key of each row's local winner: ordered fp32 bits of the logit, then
// the complement of its global index (the lowest index wins a tie, as torch.argmax)
__global__ void tp_key_kernel(const __half* __restrict__ logits, int ld, const int32_t* __restrict__ local_idx,
                              int rows, int base, unsigned long long* __restrict__ keys) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int li = local_idx[r];
  uint32_t bits = __float_as_uint(__half2float(logits[(size_t)r * ld + li]));
  if (bits == 0x80000000u) bits = 0u;  // -0 == +0: a tie, which the lower index wins
  bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
  keys[r] = ((unsigned long long)bits << 32) | (0xFFFFFFFFu - (uint32_t)(base + li));
}

__global__ void tp_key_decode_kernel(const unsigned long long* __restrict__ keys, int rows, int32_t* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) out[r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[r] & 0xFFFFFFFFull));
}

int tp_argmax(const __half* logits, int ld, int32_t* idx, int rows, int base, unsigned long long* keys, void* comm,
              cudaStream_t st) {
  tp_key_kernel<<<(rows + 127) / 128, 128, 0, st>>>(logits, ld, idx, rows, base, keys);
  if (int rc = launch_status("tp key")) return rc;
  if (int rc = tp_allreduce(comm, keys, rows, AXB_TP_MAX_U64, st)) return rc;
  tp_key_decode_kernel<<<(rows + 127) / 128, 128, 0, st>>>(keys, rows, idx);
  return launch_status("tp key decode");
}

}  // namespace axb

using namespace axb;

extern "C" {

int axb_tp_unique_id(void* id_out) {
  NcclApi& api = nccl();
  AXB_CHECK_ARG(api.ok, "tp: NCCL (libnccl.so.2) is not available");
  AXB_CHECK_ARG(id_out, "tp_unique_id: null output");
  ncclUniqueId id;
  if (int rc = nccl_status(api.get_unique_id(&id), "ncclGetUniqueId")) return rc;
  memcpy(id_out, &id, sizeof(id));
  return AXB_OK;
}

int axb_tp_comm_create(const void* id, int world, int rank, void** comm_out) {
  NcclApi& api = nccl();
  AXB_CHECK_ARG(api.ok, "tp: NCCL (libnccl.so.2) is not available");
  AXB_CHECK_ARG(id && comm_out && world >= 1 && rank >= 0 && rank < world, "tp_comm_create: bad arguments");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  if (int rc = nccl_status(api.comm_init_rank(&c, world, uid, rank), "ncclCommInitRank")) return rc;
  *comm_out = c;
  return AXB_OK;
}

int axb_tp_comm_destroy(void* comm) {
  if (!comm) return AXB_OK;
  return nccl_status(nccl().comm_destroy((ncclComm_t)comm), "ncclCommDestroy");
}

int axb_tp_comm_abort(void* comm) {
  if (!comm) return AXB_OK;
  return nccl_status(nccl().comm_abort((ncclComm_t)comm), "ncclCommAbort");
}

int axb_tp_allreduce(void* comm, void* buf_dev, size_t count, int op, void* stream) {
  return tp_allreduce(comm, buf_dev, count, op, (cudaStream_t)stream);
}

}  // extern "C"
