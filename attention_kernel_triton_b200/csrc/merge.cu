// Log-sum-exp merge of attention partials computed over disjoint key sets
// (split-KV across devices).  No reference counterpart: the reference scans a
// whole sequence in one program and stores no LSE (the LSE store is commented
// out at prefill_flash_attention.py:331-334).
//
//   O = sum_i e^{lse_i - M} O_i / sum_i e^{lse_i - M},  M = max_i lse_i
//
// Part i's outputs start at o_parts + i * o_part_stride ([rows, D] fp32,
// normalised over its own keys) and lse_parts + i * lse_part_stride ([rows]
// fp32 natural log, -inf for a part with no keys), so one all-gathered buffer
// holding [O | LSE] per device can be merged in place.  Rows with no keys
// anywhere give zeros.
#include "common.cuh"
#include "profile.cuh"

#include <cstring>
#include <string>

namespace akt {
int set_error(int code, const std::string& msg);

namespace {
template <typename T>
__global__ void __launch_bounds__(128) lse_merge_kernel(const float* __restrict__ o_parts, int64_t o_ps,
                                                        const float* __restrict__ lse_parts, int64_t l_ps, int n,
                                                        int D, T* __restrict__ out, int64_t out_row_stride) {
  const int64_t row = blockIdx.x;
  float M = -INFINITY;
  for (int i = 0; i < n; ++i) M = fmaxf(M, lse_parts[(int64_t)i * l_ps + row]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float den = 0.f, num = 0.f;
    if (M != -INFINITY) {
      for (int i = 0; i < n; ++i) {
        const float w = fast_exp2((lse_parts[(int64_t)i * l_ps + row] - M) * kLog2e);
        den += w;
        num += w * o_parts[(int64_t)i * o_ps + row * D + d];
      }
    }
    out[row * out_row_stride + d] = Elem<T>::from_float(den > 0.f ? num / den : 0.f);
  }
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Merge of the peer-stored partials: thread 0 of every CTA waits (bounded)
// until all `world` flags of this device read `epoch`, then the CTA merges its
// row from the data area; loads bypass L1 (the area is rewritten remotely).
template <typename T>
__global__ void __launch_bounds__(128) lse_merge_peer_kernel(const float* __restrict__ data, uint32_t* flags,
                                                             uint32_t* merge_counter, int world, uint32_t epoch,
                                                             int64_t rows, int D, T* __restrict__ out,
                                                             int64_t out_row_stride) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < world && ok; ++r) {
      uint32_t it = 0;
      while (ld_acquire_sys(flags + r) != epoch) {
        if ((++it & 255u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
          record_status(kStatusWaitTimeout);
          ok = 0;
          break;
        }
      }
    }
    ready = ok;
  }
  __syncthreads();
  const int64_t row = blockIdx.x;
  const int64_t part = rows * D + rows;
  float M = -INFINITY;
  if (ready)
    for (int i = 0; i < world; ++i) M = fmaxf(M, __ldcg(data + i * part + rows * D + row));
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float den = 0.f, num = 0.f;
    if (M != -INFINITY) {
      for (int i = 0; i < world; ++i) {
        const float w = fast_exp2((__ldcg(data + i * part + rows * D + row) - M) * kLog2e);
        den += w;
        num += w * __ldcg(data + i * part + row * D + d);
      }
    }
    out[row * out_row_stride + d] = Elem<T>::from_float(den > 0.f ? num / den : 0.f);
  }
  // the last CTA past its wait clears the flags for this parity's next use
  // (a writer reaches this parity again only after this kernel has finished)
  if (threadIdx.x == 0) {
    const unsigned done = atomicAdd(merge_counter, 1u) + 1u;
    if (done == gridDim.x) {
      for (int r = 0; r < world; ++r) flags[r] = 0u;
      *merge_counter = 0u;
      __threadfence();
    }
  }
}
}  // namespace
}  // namespace akt

using namespace akt;

extern "C" int akt_lse_merge_peer(const akt_peer_exchange* x, int64_t rows, int32_t head_dim, void* out,
                                  int64_t out_row_stride, int32_t dtype, void* stream) {
  if (!x || x->world < 1 || x->world > AKT_MAX_PEERS || x->rank < 0 || x->rank >= x->world || x->epoch == 0 ||
      !x->peer_data[x->rank] || !x->peer_flags[x->rank] || !x->merge_counter)
    return set_error(AKT_ERR_INVALID, "peer exchange: bad descriptor");
  if (rows < 0 || rows > 0x7fffffff || head_dim <= 0) return set_error(AKT_ERR_INVALID, "lse_merge_peer: bad sizes");
  if (dtype != AKT_FLOAT16 && dtype != AKT_BFLOAT16) return set_error(AKT_ERR_INVALID, "dtype");
  if (rows == 0) return AKT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* data = x->peer_data[x->rank];
  uint32_t* flags = x->peer_flags[x->rank];
  {
    ProfileScope prof(st);
    if (dtype == AKT_FLOAT16)
      lse_merge_peer_kernel<__half><<<(unsigned)rows, 128, 0, st>>>(data, flags, x->merge_counter, x->world,
                                                                     x->epoch, rows, head_dim,
                                                                     static_cast<__half*>(out), out_row_stride);
    else
      lse_merge_peer_kernel<__nv_bfloat16><<<(unsigned)rows, 128, 0, st>>>(
          data, flags, x->merge_counter, x->world, x->epoch, rows, head_dim, static_cast<__nv_bfloat16*>(out),
          out_row_stride);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("lse_merge_peer: ") + cudaGetErrorString(e));
  return AKT_OK;
}

// exchange regions shared between processes through CUDA IPC
extern "C" int akt_ipc_alloc(size_t bytes, void** dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out || bytes == 0) return set_error(AKT_ERR_INVALID, "ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return set_error(AKT_ERR_CUDA, std::string("ipc_alloc: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return AKT_OK;
}

extern "C" int akt_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return set_error(AKT_ERR_INVALID, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("ipc_open: ") + cudaGetErrorString(e));
  return AKT_OK;
}

extern "C" int akt_ipc_close(void* dev_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("ipc_close: ") + cudaGetErrorString(e));
  return AKT_OK;
}

extern "C" int akt_ipc_free(void* dev_ptr) {
  const cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("ipc_free: ") + cudaGetErrorString(e));
  return AKT_OK;
}

extern "C" int akt_lse_merge(const float* o_parts, int64_t o_part_stride, const float* lse_parts,
                             int64_t lse_part_stride, int32_t num_parts, int64_t rows, int32_t head_dim, void* out,
                             int64_t out_row_stride, int32_t dtype, void* stream) {
  if (num_parts < 0 || rows < 0 || head_dim <= 0) return set_error(AKT_ERR_INVALID, "lse_merge: bad sizes");
  if (dtype != AKT_FLOAT16 && dtype != AKT_BFLOAT16) return set_error(AKT_ERR_INVALID, "dtype");
  if (rows == 0) return AKT_OK;
  if (rows > 0x7fffffff) return set_error(AKT_ERR_INVALID, "lse_merge: too many rows");
  if (num_parts > 0 && (o_part_stride < rows * head_dim || lse_part_stride < rows))
    return set_error(AKT_ERR_INVALID, "lse_merge: part strides smaller than one part");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == AKT_FLOAT16)
    lse_merge_kernel<__half><<<(unsigned)rows, 128, 0, st>>>(o_parts, o_part_stride, lse_parts, lse_part_stride,
                                                             num_parts, head_dim, static_cast<__half*>(out),
                                                             out_row_stride);
  else
    lse_merge_kernel<__nv_bfloat16><<<(unsigned)rows, 128, 0, st>>>(o_parts, o_part_stride, lse_parts,
                                                                     lse_part_stride, num_parts, head_dim,
                                                                     static_cast<__nv_bfloat16*>(out),
                                                                     out_row_stride);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("lse_merge launch: ") + cudaGetErrorString(e));
  return AKT_OK;
}
