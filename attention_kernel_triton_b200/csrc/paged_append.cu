// Append new tokens' K and V rows to a paged KV cache (the write step that
// precedes the paged decodes in a serving loop; the reference has no write
// path -- its drivers build the pool in Python, decode_flash_attention_
// redundant_var_len_paged.py:337-353 and its test generators).
//
// Pool layout and page table are those of the paged decodes
// ([num_pages, 2, Hkv, P, D]; CSR indptr/indices; last_page_len).  The page
// table already covers the appended tokens: sequence b holds
// len_b = (indptr[b+1] - indptr[b] - 1) * P + last_page_len[b] tokens after
// the append, of which the last n_b = append_indptr[b+1] - append_indptr[b]
// are the new ones.  New token i of sequence b is written at position
// len_b - n_b + i: row (pos % P) of page indices[indptr[b] + pos / P].
//
// Each CTA takes 16 consecutive appended tokens: it resolves their
// destinations in parallel, then copies their K and V rows of every kv head in
// 16-byte vectors (byte work, bound by memory traffic).
// Page ids outside the pool, positions outside the sequence and malformed
// indptrs are skipped and recorded in the device status word.
#include "common.cuh"
#include "profile.cuh"

#include <string>

namespace akt {
int set_error(int code, const std::string& msg);

namespace {

struct AppendParams {
  char* cache;
  int64_t s_page, s_kv, s_head, s_tok;  // bytes
  int64_t num_pages, num_page_entries;
  const int32_t* indptr;
  const int32_t* indices;
  const int32_t* last;
  const char* k;
  const char* v;
  int64_t k_tok, k_head, v_tok, v_head;  // bytes
  const int32_t* app_indptr;
  int64_t num_append;
  int B, Hkv, P, row_bytes;
  FastDiv div_tok;   // 16-byte pieces of one token (K and V, all heads)
  FastDiv div_half;  // pieces of one token's K (or V) rows
  FastDiv div_row;   // pieces of one row
};

constexpr int kTokensPerCta = 16;
// 16-byte copies in flight per thread (cfg0's K/V, 67 MB: 19.9-20.0 us at 8,
// 20.2 at 4, 21.1 at 16)
constexpr int kPieces = 8;

// Destination row (K half; V is s_kv further) of appended token `tok`, or null
// when the page table does not place it (recorded in the status word).
__device__ __forceinline__ char* append_dst(const AppendParams& p, int64_t tok) {
  // sequence of this appended token: largest b with app_indptr[b] <= tok
  int lo = 0, hi = p.B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.app_indptr + mid) <= tok) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int a0 = __ldg(p.app_indptr + b), a1 = __ldg(p.app_indptr + b + 1);
  const int s = __ldg(p.indptr + b), e = __ldg(p.indptr + b + 1);
  if (a0 > tok || tok >= a1 || s < 0 || e <= s || e > p.num_page_entries) {
    record_status(kStatusBadIndptr);
    return nullptr;
  }
  const int last = __ldg(p.last + b);
  const int64_t len = (int64_t)(e - s - 1) * p.P + last;
  const int64_t pos = len - (a1 - a0) + (tok - a0);
  if (last < 1 || last > p.P || pos < 0 || pos >= len) {
    record_status(kStatusBadToken);
    return nullptr;
  }
  const int page = __ldg(p.indices + s + pos / p.P);
  if (page < 0 || page >= p.num_pages) {
    record_status(kStatusBadPage);
    return nullptr;
  }
  return p.cache + (int64_t)page * p.s_page + (pos % p.P) * p.s_tok;
}

// One CTA per 16 consecutive appended tokens: their destinations are resolved
// in parallel (one thread each: the lookups are chains of dependent loads),
// then every thread copies 16-byte pieces of all 16 tokens' rows.
__global__ void __launch_bounds__(256) append_paged_kernel(const AppendParams p) {
  __shared__ char* dst_s[kTokensPerCta];
  const int64_t t0 = (int64_t)blockIdx.x * kTokensPerCta;
  const int64_t rest = p.num_append - t0;
  const int nt = rest < kTokensPerCta ? (int)rest : kTokensPerCta;
  if (threadIdx.x < nt) dst_s[threadIdx.x] = append_dst(p, t0 + threadIdx.x);
  __syncthreads();
  // kPieces pieces per thread per round: their loads are independent and in flight together
  const int n = nt * (int)p.div_tok.d;
  for (int w0 = threadIdx.x; w0 < n; w0 += kPieces * blockDim.x) {
    uint4 val[kPieces];
    char* to[kPieces];
#pragma unroll
    for (int u = 0; u < kPieces; ++u) {
      const int w = w0 + u * blockDim.x;
      to[u] = nullptr;
      if (w >= n) continue;
      // piece -> (token, K or V, head, 16-byte column) by multiply-shift division
      const int i = (int)fdiv((uint32_t)w, p.div_tok), r0 = w - i * (int)p.div_tok.d;
      char* dst = dst_s[i];
      if (!dst) continue;
      const int kv = (int)fdiv((uint32_t)r0, p.div_half), r = r0 - kv * (int)p.div_half.d;
      const int h = (int)fdiv((uint32_t)r, p.div_row), c = r - h * (int)p.div_row.d;
      const int64_t tok = t0 + i;
      const char* src = (kv ? p.v + tok * p.v_tok + h * p.v_head : p.k + tok * p.k_tok + h * p.k_head) + c * 16;
      val[u] = __ldg(reinterpret_cast<const uint4*>(src));
      to[u] = dst + kv * p.s_kv + h * p.s_head + c * 16;
    }
#pragma unroll
    for (int u = 0; u < kPieces; ++u)
      if (to[u]) *reinterpret_cast<uint4*>(to[u]) = val[u];
  }
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace
}  // namespace akt

using namespace akt;

extern "C" int akt_append_paged_kv(const akt_append_paged_args* a, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  if (a->batch < 0 || a->num_kv_heads <= 0 || a->page_size <= 0 || a->head_dim <= 0 || a->num_append < 0)
    return set_error(AKT_ERR_INVALID, "append_paged_kv: bad sizes");
  if (a->dtype != AKT_FLOAT16 && a->dtype != AKT_BFLOAT16) return set_error(AKT_ERR_INVALID, "dtype");
  if (a->num_append == 0 || a->batch == 0) return AKT_OK;
  if (a->num_append > 0x7fffffff) return set_error(AKT_ERR_INVALID, "append_paged_kv: too many tokens");
  if (a->kv_stride_dim != 1 || a->k_stride_dim != 1 || a->v_stride_dim != 1)
    return set_error(AKT_ERR_UNSUPPORTED, "append_paged_kv: unit dim stride required");
  if ((a->head_dim * 2) % 16 || !al16(a->kv_cache) || !al16(a->append_k) || !al16(a->append_v) ||
      (a->kv_stride_page % 8) || (a->kv_stride_kv % 8) || (a->kv_stride_head % 8) || (a->kv_stride_token % 8) ||
      (a->k_stride_token % 8) || (a->k_stride_head % 8) || (a->v_stride_token % 8) || (a->v_stride_head % 8))
    return set_error(AKT_ERR_UNSUPPORTED, "append_paged_kv: 16-byte alignment required");
  AppendParams p{};
  p.cache = static_cast<char*>(a->kv_cache);
  p.s_page = a->kv_stride_page * 2;
  p.s_kv = a->kv_stride_kv * 2;
  p.s_head = a->kv_stride_head * 2;
  p.s_tok = a->kv_stride_token * 2;
  p.num_pages = a->num_pages;
  p.num_page_entries = a->num_page_entries;
  p.indptr = a->kv_page_indptr;
  p.indices = a->kv_page_indices;
  p.last = a->kv_last_page_len;
  p.k = static_cast<const char*>(a->append_k);
  p.v = static_cast<const char*>(a->append_v);
  p.k_tok = a->k_stride_token * 2;
  p.k_head = a->k_stride_head * 2;
  p.v_tok = a->v_stride_token * 2;
  p.v_head = a->v_stride_head * 2;
  p.app_indptr = a->append_indptr;
  p.num_append = a->num_append;
  p.B = a->batch;
  p.Hkv = a->num_kv_heads;
  p.P = a->page_size;
  p.row_bytes = a->head_dim * 2;
  const int vec = p.row_bytes / 16;  // 16-byte pieces per row
  if ((int64_t)2 * p.Hkv * vec * kTokensPerCta > 0x7fffffff)
    return set_error(AKT_ERR_UNSUPPORTED, "append_paged_kv: token rows too large");
  p.div_tok = make_fastdiv((uint32_t)(2 * p.Hkv * vec));
  p.div_half = make_fastdiv((uint32_t)(p.Hkv * vec));
  p.div_row = make_fastdiv((uint32_t)vec);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    ProfileScope prof(st);
    append_paged_kernel<<<(unsigned)((a->num_append + kTokensPerCta - 1) / kTokensPerCta), 256, 0, st>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("append_paged_kv: ") + cudaGetErrorString(e));
  return AKT_OK;
}
