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
}  // namespace
}  // namespace akt

using namespace akt;

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
