// Conversions between a per-(batch, head) keep mask over the tokens and the
// padded kept-index lists the sparse-token decodes take.
//
// mask -> (sparse_ind, sparse_nnz) replaces the Python loop of
// sparsetoken_decode_flash_attention_redundant.py:283-295: kept positions in
// ascending order (torch.nonzero order), the rest of the list -1, and an
// empty mask keeps token 0 (nnz = 1).  A row with more kept tokens than the
// list holds keeps the first max_kept of them and records
// kStatusListOverflow (the reference's slice assignment raises there).
//
// (sparse_ind, sparse_nnz) -> mask replaces the loop building precompute_mask
// at sparsetoken_decode_flash_attention_redundant.py:317-324: nnz 0 is read
// as 1, entries are read as Python indices (a negative entry counts from the
// end of the sequence, so the -1 padding of an empty list marks the last
// token, as that loop does), entries outside [-L, L) are skipped and recorded
// (kStatusBadToken; the reference raises IndexError).
//
// Both are byte/integer work bound by memory traffic: one CTA per row, the
// mask read (or written) in 16-byte vectors where alignment allows.
#include "common.cuh"
#include "profile.cuh"

#include <string>

namespace akt {
int set_error(int code, const std::string& msg);

namespace {

constexpr int kThreads = 1024;
constexpr int kPerThread = 16;                       // mask bytes per thread per chunk
constexpr int kChunk = kThreads * kPerThread;        // 16 KB of mask per pass

struct MaskToIndexParams {
  const uint8_t* mask;
  int64_t m_sb, m_sh;
  int32_t* ind;
  int64_t i_sb, i_sh;
  int32_t* nnz;
  int64_t n_sb, n_sh;
  int H, L, L_max, keep_first_if_empty;
};

// The 16 mask bytes at [pos, pos + 16) as a bitmask (bit k = byte k nonzero).
__device__ __forceinline__ uint32_t load_bits(const uint8_t* row, int pos, int L) {
  uint32_t bits = 0;
  const uint8_t* p = row + pos;
  if (pos + kPerThread <= L && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int b = 0; b < 4; ++b) bits |= (((w[i] >> (8 * b)) & 0xffu) != 0u ? 1u : 0u) << (4 * i + b);
  } else {
    for (int k = 0; k < kPerThread && pos + k < L; ++k) bits |= (p[k] != 0 ? 1u : 0u) << k;
  }
  return bits;
}

__global__ void __launch_bounds__(kThreads) mask_to_index_kernel(const MaskToIndexParams p) {
  __shared__ int warp_sums[kThreads / 32];
  __shared__ int chunk_total;
  const int row = blockIdx.x, b = row / p.H, h = row % p.H;
  const uint8_t* m = p.mask + (int64_t)b * p.m_sb + (int64_t)h * p.m_sh;
  int32_t* out = p.ind + (int64_t)b * p.i_sb + (int64_t)h * p.i_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int base = 0;  // kept positions before this chunk
  for (int c0 = 0; c0 < p.L; c0 += kChunk) {
    const int pos = c0 + threadIdx.x * kPerThread;
    const uint32_t bits = pos < p.L ? load_bits(m, pos, p.L) : 0u;
    const int cnt = __popc(bits);
    // block exclusive scan of cnt
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
      int wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += y;
      }
      warp_sums[lane] = wi - w;  // exclusive prefix of the warp totals
      if (lane == 31) chunk_total = wi;
    }
    __syncthreads();
    int at = base + warp_sums[warp] + incl - cnt;
    for (uint32_t rest = bits; rest; rest &= rest - 1, ++at)
      if (at < p.L_max) out[at] = pos + __ffs(rest) - 1;
    base += chunk_total;
    __syncthreads();  // warp_sums / chunk_total are rewritten by the next chunk
  }
  int kept = base;
  if (kept > p.L_max) {
    if (threadIdx.x == 0) record_status(kStatusListOverflow);
    kept = p.L_max;
  }
  if (base == 0 && p.keep_first_if_empty && p.L > 0 && p.L_max > 0) {
    if (threadIdx.x == 0) out[0] = 0;
    kept = 1;
  }
  for (int k = kept + threadIdx.x; k < p.L_max; k += kThreads) out[k] = -1;
  if (threadIdx.x == 0) p.nnz[(int64_t)b * p.n_sb + (int64_t)h * p.n_sh] = kept;
}

struct IndexToMaskParams {
  const int32_t* ind;
  int64_t i_sb, i_sh;
  const int32_t* nnz;
  int64_t n_sb, n_sh;
  uint8_t* mask;
  int64_t m_sb, m_sh;
  int H, L, L_max;
};

__global__ void __launch_bounds__(256) index_to_mask_kernel(const IndexToMaskParams p) {
  const int row = blockIdx.x, b = row / p.H, h = row % p.H;
  uint8_t* m = p.mask + (int64_t)b * p.m_sb + (int64_t)h * p.m_sh;
  // clear the row: 16-byte stores on the aligned middle, bytes at the edges
  const int head = min((int)((16u - (unsigned)(reinterpret_cast<uintptr_t>(m) & 15u)) & 15u), p.L);
  for (int k = threadIdx.x; k < head; k += blockDim.x) m[k] = 0;
  const int nvec = (p.L - head) / 16;
  for (int k = threadIdx.x; k < nvec; k += blockDim.x)
    reinterpret_cast<uint4*>(m + head)[k] = make_uint4(0, 0, 0, 0);
  for (int k = head + nvec * 16 + threadIdx.x; k < p.L; k += blockDim.x) m[k] = 0;
  __syncthreads();
  const int32_t* list = p.ind + (int64_t)b * p.i_sb + (int64_t)h * p.i_sh;
  int n = p.nnz[(int64_t)b * p.n_sb + (int64_t)h * p.n_sh];
  if (n == 0) n = 1;
  n = min(n, p.L_max);  // a Python slice stops at the list end
  for (int k = threadIdx.x; k < n; k += blockDim.x) {
    int t = list[k];
    if (t < 0) t += p.L;
    if (t < 0 || t >= p.L) {
      record_status(kStatusBadToken);
      continue;
    }
    m[t] = 1;
  }
}

}  // namespace
}  // namespace akt

using namespace akt;

extern "C" int akt_mask_to_sparse_index(const akt_mask_to_index_args* a, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  if (a->batch < 0 || a->num_heads < 0 || a->seq_len < 0 || a->max_kept < 0)
    return set_error(AKT_ERR_INVALID, "mask_to_sparse_index: sizes must be non-negative");
  if ((int64_t)a->batch * a->num_heads > 0x7fffffff)
    return set_error(AKT_ERR_INVALID, "mask_to_sparse_index: too many rows");
  if (a->batch == 0 || a->num_heads == 0) return AKT_OK;
  if (!a->mask || !a->sparse_nnz || (!a->sparse_ind && a->max_kept > 0))
    return set_error(AKT_ERR_INVALID, "mask_to_sparse_index: null pointer");
  MaskToIndexParams p{};
  p.mask = a->mask;
  p.m_sb = a->mask_stride_batch;
  p.m_sh = a->mask_stride_head;
  p.ind = a->sparse_ind;
  p.i_sb = a->ind_stride_batch;
  p.i_sh = a->ind_stride_head;
  p.nnz = a->sparse_nnz;
  p.n_sb = a->nnz_stride_batch;
  p.n_sh = a->nnz_stride_head;
  p.H = a->num_heads;
  p.L = a->seq_len;
  p.L_max = a->max_kept;
  p.keep_first_if_empty = a->keep_first_if_empty ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    ProfileScope prof(st);
    mask_to_index_kernel<<<(unsigned)(a->batch * a->num_heads), kThreads, 0, st>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("mask_to_sparse_index: ") + cudaGetErrorString(e));
  return AKT_OK;
}

extern "C" int akt_sparse_index_to_mask(const akt_index_to_mask_args* a, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  if (a->batch < 0 || a->num_heads < 0 || a->seq_len < 0 || a->max_kept < 0)
    return set_error(AKT_ERR_INVALID, "sparse_index_to_mask: sizes must be non-negative");
  if ((int64_t)a->batch * a->num_heads > 0x7fffffff)
    return set_error(AKT_ERR_INVALID, "sparse_index_to_mask: too many rows");
  if (a->batch == 0 || a->num_heads == 0 || a->seq_len == 0) return AKT_OK;
  if (!a->mask || !a->sparse_nnz || (!a->sparse_ind && a->max_kept > 0))
    return set_error(AKT_ERR_INVALID, "sparse_index_to_mask: null pointer");
  IndexToMaskParams p{};
  p.ind = a->sparse_ind;
  p.i_sb = a->ind_stride_batch;
  p.i_sh = a->ind_stride_head;
  p.nnz = a->sparse_nnz;
  p.n_sb = a->nnz_stride_batch;
  p.n_sh = a->nnz_stride_head;
  p.mask = a->mask;
  p.m_sb = a->mask_stride_batch;
  p.m_sh = a->mask_stride_head;
  p.H = a->num_heads;
  p.L = a->seq_len;
  p.L_max = a->max_kept;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    ProfileScope prof(st);
    index_to_mask_kernel<<<(unsigned)(a->batch * a->num_heads), 256, 0, st>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("sparse_index_to_mask: ") + cudaGetErrorString(e));
  return AKT_OK;
}
