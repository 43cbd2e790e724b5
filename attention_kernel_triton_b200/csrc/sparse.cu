// Sparse-token GQA decode for sm_100a: dense KV, paged KV, and MagicPIG.
//
// Replaces the Triton kernels of
//   sparsetoken_decode_flash_attention_redundant.py:11-124            (dense KV)
//   sparsetoken_decode_flash_attention_redundant_var_len_paged.py:11-167  (paged KV)
//   magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_with_norm.py:16-164
// Same math: softmax over the kept tokens sparse_ind[b, h, 0:nnz) only (SD:81-121);
// paged tokens resolved through the CSR page table (SP:114-126); MagicPIG
// scores q.k/sqrt(D) - log(u) with u from the LSH collision probability of
// cos(q, k) (MP:110-148, with the naive reference's clamps, MP:263-278).
//
// Machine mapping:
//  * Work item = (sequence, kv head, group of G qo heads, 32 consecutive list
//    positions).  A one-CTA planner turns nnz into per-unit chunk counts and
//    offsets; persistent CTAs walk the item list; a merge kernel combines the
//    per-chunk (O, log2-sum-exp) partials of each head.
//  * Gather: 32 threads resolve one kept row each to an element offset (the
//    page-table lookup for paged K/V); then all threads load the rows' 16-byte
//    pieces with streaming loads into shared memory.
//  * GQA: the index lists are per qo head in the API.  When the G heads of an
//    item carry identical positions (the common case: a per-kv-head keep mask
//    repeated over the group) the rows are gathered once and all G heads are
//    computed from them; otherwise each head gathers its own rows.
//  * Compute: the shared warp core (attn_core.cuh), CUDA cores only.
#include "attn_core.cuh"
#include "common.cuh"
#include "profile.cuh"

#include <algorithm>
#include <string>

namespace akt {

int set_error(int code, const std::string& msg);
int sm_count();

namespace {

constexpr int kSW = 4;             // warps per CTA
constexpr int kSThreads = 32 * kSW;
constexpr int kCP = 32;            // list positions per work item
constexpr float kPi = 3.14159265358979323846f;

struct SparseParams {
  const void* q;
  int64_t q_sb, q_sh;
  const void* k;  // dense: K base; paged: pool base
  const void* v;  // dense: V base; paged: pool base + stride_kv
  int64_t s0, s_head, s_tok;  // dense: batch/head/token strides; paged: page/head/token
  const int32_t* indptr;
  const int32_t* indices;
  int64_t num_pages, num_page_entries;
  const int32_t* ind;
  int64_t ind_sb, ind_sh, ind_sp;
  const int32_t* nnz;
  int64_t nnz_sb, nnz_sh;
  // CSR lists (instead of ind/nnz): row r = b * Hq + h holds
  // ind[csr_ptr[r] .. csr_ptr[r + 1]) of a flat index array of num_inds entries
  const int32_t* csr_ptr;
  int64_t num_inds;
  const float* mp_k;
  const float* mp_l;
  int64_t par_sb, par_sh;
  void* out;
  int64_t o_sb, o_sh, o_sd;
  int B, Hq, Hkv, L, P, max_nnz;
  int group, g_tiles, units;  // units per batch = Hkv * g_tiles
  float scale_log2;
  float inv_sqrt_d;
  float* part_o;       // [items, G, D]
  float* part_lse;     // [items, G]
  int* unit_offset;    // [B * units + 1]
  // partial-output mode (KV split across devices): when set, the merge writes
  // the fp32 normalised O [B, Hq, D] and natural-log LSE [B, Hq] of this
  // device's tokens instead of the typed output
  float* out_part_o;
  float* out_part_lse;
  // peer-store exchange (partial mode): the merge also stores each partial
  // row into slot `rank` of every device's data area and, when all its CTAs
  // are done, raises flag `rank` on every device
  int inline_plan;  // B * units <= kSThreads: every CTA computes the unit offsets itself (no planner)
  int n_peers, rank;
  uint32_t epoch;
  float* peer_data[AKT_MAX_PEERS];
  uint32_t* peer_flags[AKT_MAX_PEERS];
  uint32_t* counter;
  // fused final merge (akt_sparse_dense_split_peer): after publishing, every
  // merge CTA waits for all ranks' flags on this device and merges its own
  // rows of the data area into the typed output
  int final_merge;
  uint32_t* merge_counter;
};

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------
// planner: chunks per (batch, unit) = ceil(max nnz over the unit's heads / kCP)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int clamped_nnz(const SparseParams& p, int b, int h) {
  int n;
  if (p.csr_ptr) {
    const int64_t r = (int64_t)b * p.Hq + h;
    const int s = __ldg(p.csr_ptr + r), e = __ldg(p.csr_ptr + r + 1);
    if (s < 0 || e < s || e > p.num_inds) {  // malformed row offsets: the row keeps nothing
      record_status(kStatusBadIndptr);
      return 0;
    }
    n = e - s;
  } else {
    n = p.nnz[(int64_t)b * p.nnz_sb + (int64_t)h * p.nnz_sh];
  }
  if (n > p.max_nnz) {
    record_status(kStatusBadToken);
    n = p.max_nnz;
  }
  return n < 0 ? 0 : n;
}

template <int G>
__global__ void __launch_bounds__(1024) sparse_plan_kernel(SparseParams p) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_units = p.B * p.units;
  for (int base = 0; base < n_units; base += 1024) {
    const int u = base + threadIdx.x;
    int n = 0;
    if (u < n_units) {
      const int b = u / p.units, unit = u - b * p.units;
      const int kvh = unit / p.g_tiles;
      const int head0 = kvh * p.group + (unit - kvh * p.g_tiles) * G;
      int mx = 0;
      for (int h = 0; h < G; ++h) mx = max(mx, clamped_nnz(p, b, head0 + h));
      n = cdiv(mx, kCP);
    }
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (u < n_units) p.unit_offset[u] = carry + incl - n;
    __syncthreads();
    if (threadIdx.x == 1023) carry += incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) p.unit_offset[n_units] = carry;
}

// ---------------------------------------------------------------------------
// scores
// ---------------------------------------------------------------------------
struct MagicPigScore {
  float qn;       // |q| of the lane's head
  float K, Lp;    // LSH parameters of the lane's head
  float inv_sqrt_d;
  __device__ __forceinline__ float operator()(float dot, float kk, int) const {
    const float kn = sqrtf(kk);
    float c = dot / (qn * kn + 1e-8f);
    c = fminf(fmaxf(c, -1.0f + 1e-7f), 1.0f - 1e-7f);
    float pr = 1.0f - (1.0f / kPi) * acosf(c);
    pr = fminf(fmaxf(pr, 0.0f), 1.0f);
    // p^K and (1-p^K)^(L-1) as exp2(e * log2(base)) through CUDA's exp2f and
    // log2f, and (1-p^K)^L as (1-p^K) * (1-p^K)^(L-1): one logarithm and one
    // exponential per power instead of three powf calls.  A zero base keeps
    // powf, for its special cases (0^0 = 1, 0 to a negative power).
    const float pK = pr > 0.f ? exp2f(K * log2f(pr)) : powf(pr, K);
    const float omp = fminf(fmaxf(1.0f - pK, 0.0f), 1.0f);
    float u;
    if (omp > 0.f) {
      const float y = exp2f((Lp - 1.0f) * log2f(omp));  // (1-p^K)^(L-1)
      u = 1.0f - y * (omp + Lp * pK);
    } else {
      u = 1.0f - powf(omp, Lp) - Lp * pK * powf(omp, Lp - 1.0f);
    }
    u = fmaxf(u, 1e-10f);
    return (dot * inv_sqrt_d - logf(u)) * kLog2e;
  }
};

// ---------------------------------------------------------------------------
// shared-memory layout of one CTA
// ---------------------------------------------------------------------------
template <typename T, int D, int G>
struct SparseSmem {
  static constexpr size_t kv = (size_t)2 * kCP * D * sizeof(T);
  static constexpr size_t comb = sizeof(float) * ((size_t)kSW * G * (2 + D) + (size_t)kSW * kRowsPerSubTile * G);
  static constexpr size_t idx = sizeof(int) * ((size_t)G * kCP + G + 4);
  static constexpr size_t flags = 64;  // kCP row-valid bytes, padded
  static constexpr size_t offs = sizeof(int64_t) * kCP;  // element offset of each gathered row
  static constexpr size_t bytes = kv + comb + idx + flags + offs + 16;
};

template <typename T, int D, int G, bool PAGED, bool MAGIC>
struct SparseCta {
  using E = Elem<T>;
  const SparseParams& p;
  T* Ks;
  T* Vs;
  float *comb_m, *comb_l, *comb_o, *p_s;
  int* idx_s;
  int* nnz_s;
  int* item_s;  // [0] unit, [1] chunk of the current item, [2..3] indptr[b], indptr[b + 1]
  unsigned char* ok_s;
  int64_t* off_s;
  uint64_t* bar;
  int tid, warp, lane;
  uint32_t phase;
  uint64_t pol;

  __device__ SparseCta(const SparseParams& p_, unsigned char* smem) : p(p_) {
    Ks = reinterpret_cast<T*>(smem);
    Vs = Ks + kCP * D;
    comb_m = reinterpret_cast<float*>(smem + SparseSmem<T, D, G>::kv);
    comb_l = comb_m + kSW * G;
    comb_o = comb_l + kSW * G;
    p_s = comb_o + kSW * G * D;
    idx_s = reinterpret_cast<int*>(p_s + kSW * kRowsPerSubTile * G);
    nnz_s = idx_s + G * kCP;
    item_s = nnz_s + G;
    ok_s = reinterpret_cast<unsigned char*>(item_s + 4);
    off_s = reinterpret_cast<int64_t*>((reinterpret_cast<uintptr_t>(ok_s + 64) + 7) & ~uintptr_t(7));
    bar = reinterpret_cast<uint64_t*>(off_s + kCP);
    tid = threadIdx.x;
    warp = tid >> 5;
    lane = tid & 31;
    phase = 0;
    pol = l2_policy_evict_first();
  }

  // Gather the K/V rows of list positions rows[0..kCP) (token ids, -1 = none)
  // into Ks/Vs.  Invalid rows are zero-filled and flagged in ok_s.
  // The first kCP threads resolve their row's element offset (the page-table
  // lookup for paged K/V); then every thread loads 16-byte pieces of the rows
  // with plain streaming loads, all of a thread's loads issued before its
  // shared-memory stores.  (One 1-D bulk copy per 512-byte row took about
  // twice as long: 64 small copies per item through the TMA engine.)
  __device__ bool gather(const int* rows, int b, int kvh) {
    if (tid < kCP) {
      bool ok = false;
      int64_t off = 0;
      const int tok = rows[tid];
      if (tok >= 0) {
        if (PAGED) {
          const int s = item_s[2], e = item_s[3];  // indptr[b], indptr[b + 1]
          const int npg = e - s;
          if (s < 0 || npg < 0 || e > p.num_page_entries || tok >= npg * p.P) {
            record_status(kStatusBadToken);
          } else {
            const int pg = tok / p.P;
            const int phys = __ldg(p.indices + s + pg);
            if (phys < 0 || (int64_t)phys >= p.num_pages) {
              record_status(kStatusBadPage);
            } else {
              ok = true;
              off = (int64_t)phys * p.s0 + (int64_t)kvh * p.s_head + (int64_t)(tok - pg * p.P) * p.s_tok;
            }
          }
        } else {
          if (tok >= p.L) {
            record_status(kStatusBadToken);
          } else {
            ok = true;
            off = (int64_t)b * p.s0 + (int64_t)kvh * p.s_head + (int64_t)tok * p.s_tok;
          }
        }
      }
      ok_s[tid] = ok ? 1 : 0;
      off_s[tid] = ok ? off : -1;
    }
    __syncthreads();
    constexpr int kPiecesPerRow = D * (int)sizeof(T) / 16;
    constexpr int kPieces = kCP * kPiecesPerRow;  // per matrix
    constexpr int kPerThread = kPieces / kSThreads;
    static_assert(kPieces % kSThreads == 0, "pieces per thread");
    constexpr int kBatch = kPerThread > 4 ? 4 : kPerThread;  // loads in flight per batch (x2: K and V)
    const uint4* kb = static_cast<const uint4*>(p.k);
    const uint4* vb = static_cast<const uint4*>(p.v);
    uint4* kd = reinterpret_cast<uint4*>(Ks);
    uint4* vd = reinterpret_cast<uint4*>(Vs);
#pragma unroll
    for (int i0 = 0; i0 < kPerThread; i0 += kBatch) {
      uint4 kr[kBatch], vr[kBatch];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int e = tid + (i0 + i) * kSThreads;
        const int r = e / kPiecesPerRow, c = e - r * kPiecesPerRow;
        const int64_t o = off_s[r];
        if (o >= 0) {
          kr[i] = __ldcs(kb + o / 8 + c);
          vr[i] = __ldcs(vb + o / 8 + c);
        } else {
          kr[i] = make_uint4(0, 0, 0, 0);
          vr[i] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int e = tid + (i0 + i) * kSThreads;
        kd[e] = kr[i];
        vd[e] = vr[i];
      }
    }
    __syncthreads();
    return true;
  }

  // attention of NH heads (head0 + hoff ...) over the gathered rows; writes
  // the partial of item `item` at head slot hoff.
  template <int NH>
  __device__ void compute(int item, int b, int head_first, int hoff) {
    WarpAttn<T, D, NH, MAGIC> wa;
    wa.init(lane);
    const T* q0 = static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)head_first * p.q_sh;
    wa.load_q(q0, p.q_sh, MAGIC ? 1.0f : p.scale_log2);
    constexpr int RPW = kCP / kSW;  // rows per warp
    const int row0 = warp * RPW;
    const uint32_t bits = __ballot_sync(0xffffffffu, lane < RPW && ok_s[row0 + min(lane, RPW - 1)]);
    float* pw = p_s + warp * kRowsPerSubTile * G;
    if constexpr (MAGIC) {
      const int hq = head_first + wa.my_head;
      MagicPigScore sc;
      sc.qn = sqrtf(wa.q_norm2_my_head());
      sc.K = p.mp_k[(int64_t)b * p.par_sb + (int64_t)hq * p.par_sh];
      sc.Lp = p.mp_l[(int64_t)b * p.par_sb + (int64_t)hq * p.par_sh];
      sc.inv_sqrt_d = p.inv_sqrt_d;
      wa.template step<true>(Ks, Vs, row0, RPW, kCP - 1, bits, pw, sc);
    } else {
      wa.template step<true>(Ks, Vs, row0, RPW, kCP - 1, bits, pw, ScaledDotScore());
    }
    wa.stash(comb_m, comb_l, comb_o, warp, true);
    __syncthreads();
    for (int e = tid; e < NH * D; e += kSThreads) {
      const int h = e / D, d = e - h * D;
      float lse2;
      const float val = combine_warps<kSW, NH, D>(comb_m, comb_l, comb_o, h, d, lse2);
      p.part_o[((int64_t)item * G + hoff + h) * D + d] = val;
      if (d == 0) p.part_lse[(int64_t)item * G + hoff + h] = lse2;
    }
    __syncthreads();
  }
};

template <typename T, int D, int G, bool PAGED, bool MAGIC>
__global__ void __launch_bounds__(kSThreads, MAGIC ? 3 : 4) sparse_decode_kernel(const SparseParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  SparseCta<T, D, G, PAGED, MAGIC> cta(p, smem);
  if (cta.tid == 0) {
    mbar_init(cta.bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int n_units = p.B * p.units;
  // unit offsets (items per unit = ceil(max nnz of its heads / kCP), exclusive
  // prefix): from the planner kernel, or for a few units computed here by
  // every CTA (one thread per unit), which takes a launch off short calls;
  // CTA 0 then also stores them for the merge kernel
  __shared__ int uoff_s[kSThreads + 1];
  int total;
  if (p.inline_plan) {
    const int t = cta.tid;
    int n = 0;
    if (t < n_units) {
      const int bb = t / p.units, un = t - bb * p.units;
      const int kv = un / p.g_tiles;
      const int h0 = kv * p.group + (un - kv * p.g_tiles) * G;
      int mx = 0;
      for (int h = 0; h < G; ++h) mx = max(mx, clamped_nnz(p, bb, h0 + h));
      n = cdiv(mx, kCP);
    }
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (cta.lane >= o) x += y;
    }
    if (cta.lane == 31) cta.idx_s[cta.warp] = x;  // warp totals (idx_s is free until the first item)
    __syncthreads();
    int before = 0;
    for (int w = 0; w < cta.warp; ++w) before += cta.idx_s[w];
    const int incl = x + before;
    uoff_s[t] = incl - n;
    if (t == kSThreads - 1) uoff_s[kSThreads] = incl;
    __syncthreads();
    if (t > n_units) uoff_s[t] = uoff_s[kSThreads];  // past the last unit: the total
    if (t == 0) uoff_s[n_units] = uoff_s[kSThreads];
    __syncthreads();
    if (blockIdx.x == 0 && t <= n_units) p.unit_offset[t] = uoff_s[t];
    total = uoff_s[n_units];
  } else {
    grid_dep_wait();  // item offsets come from the planner kernel
    total = p.unit_offset[n_units];
  }
  const int* uoff = p.inline_plan ? uoff_s : p.unit_offset;
  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    // The item's unit u: the one with unit_offset[u] <= item < unit_offset[u + 1].
    // Up to kSThreads units: one round of independent loads, one thread per
    // unit (exactly one matches; units with no items have equal bounds).
    // More units: binary search.  The loads that follow are issued together
    // where they do not depend on each other: each is a round trip to memory,
    // and one item per CTA (short lists) is a handful of them end to end.
    if (n_units <= kSThreads) {
      if (cta.tid < n_units) {
        const int a = uoff[cta.tid], z = uoff[cta.tid + 1];
        if (a <= item && item < z) {
          cta.item_s[0] = cta.tid;
          cta.item_s[1] = item - a;
        }
      }
    } else if (cta.tid == 0) {
      int lo = 0, hi = n_units - 1;  // largest u with unit_offset[u] <= item
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.unit_offset[mid] <= item) lo = mid; else hi = mid - 1;
      }
      cta.item_s[0] = lo;
      cta.item_s[1] = item - p.unit_offset[lo];
    }
    __syncthreads();
    const int u = cta.item_s[0];
    const int c = cta.item_s[1];
    const int b = u / p.units, unit = u - b * p.units;
    const int kvh = unit / p.g_tiles;
    const int head0 = kvh * p.group + (unit - kvh * p.g_tiles) * G;
    const int p0 = c * kCP;
    // first load round: nnz (CSR: row offsets), the page range (paged) and, for padded
    // lists, the list entries themselves (positions < max_nnz exist; those
    // at or past nnz are masked once nnz is known)
    if (cta.tid < G) cta.nnz_s[cta.tid] = clamped_nnz(p, b, head0 + cta.tid);
    if (PAGED && cta.tid == G) {
      cta.item_s[2] = p.indptr[b];
      cta.item_s[3] = p.indptr[b + 1];
    }
    if (!p.csr_ptr) {
      for (int e = cta.tid; e < G * kCP; e += kSThreads) {
        const int h = e / kCP, j = e - h * kCP;
        const int pos = p0 + j;
        cta.idx_s[e] = pos < p.max_nnz
                           ? p.ind[(int64_t)b * p.ind_sb + (int64_t)(head0 + h) * p.ind_sh + (int64_t)pos * p.ind_sp]
                           : -1;
      }
    }
    __syncthreads();
    // second load round: CSR entries (their row offset is checked by clamped_nnz, nnz 0
    // if malformed); padded entries past nnz masked (each thread its own)
    for (int e = cta.tid; e < G * kCP; e += kSThreads) {
      const int h = e / kCP, j = e - h * kCP;
      const int pos = p0 + j;
      if (pos >= cta.nnz_s[h])
        cta.idx_s[e] = -1;
      else if (p.csr_ptr)
        cta.idx_s[e] = p.ind[(int64_t)__ldg(p.csr_ptr + (int64_t)b * p.Hq + head0 + h) + pos];
    }
    __syncthreads();
    bool same = true;
    for (int e = cta.tid; e < (G - 1) * kCP; e += kSThreads) same &= cta.idx_s[kCP + e] == cta.idx_s[e % kCP];
    const bool packed = __syncthreads_and(same) != 0;
    if (packed) {
      if (!cta.gather(cta.idx_s, b, kvh)) return;
      cta.template compute<G>(item, b, head0, 0);
    } else {
      for (int h = 0; h < G; ++h) {
        if (!cta.gather(cta.idx_s + h * kCP, b, kvh)) return;
        cta.template compute<1>(item, b, head0 + h, h);
      }
    }
  }
}

// four floats to dst: one 16-byte store where dst is 16-byte aligned (a
// partial row's start is not, when B * Hq is not a multiple of 4)
__device__ __forceinline__ void store4(float* dst, float4 v) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    *reinterpret_cast<float4*>(dst) = v;
  } else {
    dst[0] = v.x;
    dst[1] = v.y;
    dst[2] = v.z;
    dst[3] = v.w;
  }
}

// merge of the per-chunk partials of every (batch, unit): chunks are the
// contiguous items unit_offset[u] .. unit_offset[u+1).  Per head, one warp
// takes the max and the sum of 2^(lse - max) over the chunks (lanes striding
// the chunks).  Then the NT threads form NT / (G * D / 4) groups; in each group
// a thread accumulates four consecutive dims of one head over every
// groups-th chunk (one 16-byte load per chunk, unrolled so several loads are
// in flight), and the groups' sums are added in shared memory.  NT = 1024 on
// the single-device path when the (batch, unit) pairs fit one wave (their
// chunk lists are then long: ~80 per pair for one 128K sequence); 256
// otherwise, and always with the peer exchange, whose fused final merge
// relies on four CTAs of this kernel being resident per SM.
template <typename T, int D, int G, int NT>
__global__ void __launch_bounds__(NT, NT == 256 ? 4 : 1) sparse_merge_kernel(const SparseParams p) {
  using E = Elem<T>;
  grid_dep_wait();  // partials (and item offsets) of the previous kernels
  const int u = blockIdx.x;
  const int b = u / p.units, unit = u - b * p.units;
  const int kvh = unit / p.g_tiles;
  const int head0 = kvh * p.group + (unit - kvh * p.g_tiles) * G;
  const int i0 = p.unit_offset[u], i1 = p.unit_offset[u + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float head_m[G], head_den[G];
  constexpr int NE = G * D / 4;  // four-dim elements of the unit's output
  static_assert(NT % NE == 0, "groups");
  constexpr int kGroups = NT / NE;
  __shared__ float4 red[kGroups > 1 ? (kGroups - 1) * NE : 1];  // sums of groups 1..
  for (int h = warp; h < G; h += NT / 32) {
    float m = -INFINITY;
    for (int it = i0 + lane; it < i1; it += 32) m = fmaxf(m, p.part_lse[(int64_t)it * G + h]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float den = 0.f;
    if (m != -INFINITY)
      for (int it = i0 + lane; it < i1; it += 32) den += fast_exp2(p.part_lse[(int64_t)it * G + h] - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (lane == 0) {
      head_m[h] = m;
      head_den[h] = den;
    }
  }
  __syncthreads();
  T* out = static_cast<T*>(p.out);
  const int64_t rows = (int64_t)p.B * p.Hq;
  const int gi = threadIdx.x / NE, e4 = threadIdx.x - gi * NE;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
  {
    const int h = (4 * e4) / D, d = 4 * e4 - h * D;
    const float M = head_m[h];
    if (M != -INFINITY) {
#pragma unroll 8
      for (int it = i0 + gi; it < i1; it += kGroups) {
        const float w = fast_exp2(p.part_lse[(int64_t)it * G + h] - M);
        const float4 o = *reinterpret_cast<const float4*>(p.part_o + ((int64_t)it * G + h) * D + d);
        num.x += w * o.x;
        num.y += w * o.y;
        num.z += w * o.z;
        num.w += w * o.w;
      }
    }
    if (kGroups > 1 && gi > 0) red[(gi - 1) * NE + e4] = num;
  }
  if (kGroups > 1) __syncthreads();
  if (gi == 0) {
    const int h = (4 * e4) / D, d = 4 * e4 - h * D;
    const float M = head_m[h], den = head_den[h];
#pragma unroll
    for (int g2 = 1; g2 < kGroups; ++g2) {
      const float4 o = red[(g2 - 1) * NE + e4];
      num.x += o.x;
      num.y += o.y;
      num.z += o.z;
      num.w += o.w;
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    const float4 val = make_float4(num.x * inv, num.y * inv, num.z * inv, num.w * inv);
    const int64_t row = (int64_t)b * p.Hq + head0 + h;
    if (p.n_peers) {
      const float lse = den > 0.f ? (M + log2f(den)) * kLn2 : -INFINITY;
      for (int r = 0; r < p.n_peers; ++r) {
        float* slot = p.peer_data[r] + (int64_t)p.rank * (rows * D + rows);
        store4(slot + row * D + d, val);
        if (d == 0) slot[rows * D + row] = lse;
      }
    } else if (p.out_part_o) {
      store4(p.out_part_o + row * D + d, val);
      if (d == 0) p.out_part_lse[row] = den > 0.f ? (M + log2f(den)) * kLn2 : -INFINITY;
    } else {
      T* orow = out + (int64_t)b * p.o_sb + (int64_t)(head0 + h) * p.o_sh;
      orow[(int64_t)d * p.o_sd] = E::from_float(val.x);
      orow[(int64_t)(d + 1) * p.o_sd] = E::from_float(val.y);
      orow[(int64_t)(d + 2) * p.o_sd] = E::from_float(val.z);
      orow[(int64_t)(d + 3) * p.o_sd] = E::from_float(val.w);
    }
  }
  if (p.n_peers) {
    // every thread's stores are visible system-wide before this CTA counts
    // itself done; the last CTA raises the flags (the counter resets for the
    // next call, which is stream-ordered after this kernel)
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned done = atomicAdd(p.counter, 1u) + 1u;
      if (done == gridDim.x) {
        __threadfence_system();
        for (int r = 0; r < p.n_peers; ++r) st_release_sys(p.peer_flags[r] + p.rank, p.epoch);
        *p.counter = 0u;
      }
    }
    if (p.final_merge) {
      // wait (bounded) until every rank's partial has landed in this device's
      // data area; every CTA of this grid is resident (the host launches this
      // form only for a grid that fits at once), so the last one to count
      // itself in above is never held back by a waiting one
      const uint32_t* flags = p.peer_flags[p.rank];
      __shared__ int ready;
      if (threadIdx.x == 0) {
        int ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int r = 0; r < p.n_peers && ok; ++r) {
          uint32_t spins = 0;
          while (ld_acquire_sys_u32(flags + r) != p.epoch) {
            if ((++spins & 255u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
              record_status(kStatusWaitTimeout);
              ok = 0;
              break;
            }
          }
        }
        ready = ok;
      }
      __syncthreads();
      // O = sum_r e^{lse_r - M} O_r / sum_r e^{lse_r - M} for this unit's rows
      // (L2 loads: the area is written over NVLink)
      const float* area = p.peer_data[p.rank];
      const int64_t part = rows * D + rows;
      for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
        const int h = e / D, d = e - h * D;
        const int64_t row = (int64_t)b * p.Hq + head0 + h;
        float M = -INFINITY;
        if (ready)
          for (int r = 0; r < p.n_peers; ++r) M = fmaxf(M, __ldcg(area + r * part + rows * D + row));
        float den = 0.f, num = 0.f;
        if (M != -INFINITY) {
          for (int r = 0; r < p.n_peers; ++r) {
            const float w = fast_exp2((__ldcg(area + r * part + rows * D + row) - M) * kLog2e);
            den += w;
            num += w * __ldcg(area + r * part + row * D + d);
          }
        }
        out[(int64_t)b * p.o_sb + (int64_t)(head0 + h) * p.o_sh + (int64_t)d * p.o_sd] =
            E::from_float(den > 0.f ? num / den : 0.f);
      }
      // the last CTA past its wait clears this device's flags for the parity's
      // next use (a writer reaches this parity again only after this kernel)
      __syncthreads();
      if (threadIdx.x == 0) {
        const unsigned fin = atomicAdd(p.merge_counter, 1u) + 1u;
        if (fin == gridDim.x) {
          for (int r = 0; r < p.n_peers; ++r) p.peer_flags[p.rank][r] = 0u;
          *p.merge_counter = 0u;
          __threadfence();
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
struct SparsePlan {
  int G_tile, units;
  int64_t items;  // upper bound
  size_t smem, ws_bytes, off_lse, off_units;
};

int sparse_group_tile(int group, int D) {
  const int cap = D >= 256 ? 4 : 8;
  for (int g = cap; g >= 2; g >>= 1)
    if (group % g == 0) return g;
  return 1;
}

size_t al256(size_t x) { return (x + 255) / 256 * 256; }

template <typename T, int D, int G>
size_t sparse_smem_bytes() {
  return SparseSmem<T, D, G>::bytes;
}

SparsePlan make_sparse_plan(int B, int Hq, int Hkv, int D, int max_nnz) {
  SparsePlan pl{};
  const int group = Hq / Hkv;
  pl.G_tile = sparse_group_tile(group, D);
  pl.units = Hkv * (group / pl.G_tile);
  pl.items = (int64_t)B * pl.units * cdiv(std::max(max_nnz, 0), kCP);
  size_t ws = al256((size_t)std::max<int64_t>(pl.items, 1) * pl.G_tile * D * sizeof(float));
  pl.off_lse = ws;
  ws += al256((size_t)std::max<int64_t>(pl.items, 1) * pl.G_tile * sizeof(float));
  pl.off_units = ws;
  ws += al256(((size_t)B * pl.units + 1) * sizeof(int));
  pl.ws_bytes = ws;
  return pl;
}

template <typename T, int D, int G, bool PAGED, bool MAGIC>
int launch_sparse(const SparseParams& p, const SparsePlan& pl, cudaStream_t st) {
  auto kern = sparse_decode_kernel<T, D, G, PAGED, MAGIC>;
  const size_t smem = SparseSmem<T, D, G>::bytes;
  cudaError_t e;
  if (p.final_merge && p.B * p.units > 0) {
    // the fused final merge waits on its own grid: every CTA must be resident
    // (checked before anything is launched, so a refusal leaves no partial
    // exchange behind)
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sparse_merge_kernel<T, D, G, 256>, 256, 0);
    if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(e));
    if ((int64_t)p.B * p.units > (int64_t)per_sm * sm_count())
      return set_error(AKT_ERR_UNSUPPORTED, "split_peer: the merge grid does not fit the GPU at once");
  }
  e = ensure_smem_limit<sparse_decode_kernel<T, D, G, PAGED, MAGIC>>(smem);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  // One resident wave of CTAs walks the items (the count is an upper bound
  // from the list capacity; the planner finds the real one on the device).
  // CTAs beyond what fits would wait for a second wave, mostly to find no
  // item.  Residency per SM is read once per instantiation.
  static const int resident = [&] {
    int n = 0;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kSThreads, smem) == cudaSuccess && n > 0 ? n : 1;
  }();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(pl.items, (int64_t)sm_count() * resident));
  if (p.inline_plan && pl.items > 0) {
    // first kernel of the call (reads the caller's inputs): launched normally
    ProfileScope prof(st);
    kern<<<grid, kSThreads, smem, st>>>(p);
  } else {
    sparse_plan_kernel<G><<<1, 1024, 0, st>>>(p);
    if (pl.items > 0) {
      ProfileScope prof(st);
      e = launch_dependent(kern, dim3(grid), dim3(kSThreads), smem, st, p);
      if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("sparse launch: ") + cudaGetErrorString(e));
    }
  }
  const unsigned nb = (unsigned)(p.B * p.units);
  if (nb > 0) {
    if (!p.n_peers && nb <= (unsigned)sm_count())
      e = launch_dependent(sparse_merge_kernel<T, D, G, 1024>, dim3(nb), dim3(1024), 0, st, p);
    else
      e = launch_dependent(sparse_merge_kernel<T, D, G, 256>, dim3(nb), dim3(256), 0, st, p);
  }
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("sparse merge launch: ") + cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("sparse launch: ") + cudaGetErrorString(e));
  return AKT_OK;
}

template <typename T, bool PAGED, bool MAGIC>
int dispatch_sparse(const SparseParams& p, const SparsePlan& pl, int D, cudaStream_t st) {
  switch (D) {
    case 64:
      switch (pl.G_tile) {
        case 1: return launch_sparse<T, 64, 1, PAGED, MAGIC>(p, pl, st);
        case 2: return launch_sparse<T, 64, 2, PAGED, MAGIC>(p, pl, st);
        case 4: return launch_sparse<T, 64, 4, PAGED, MAGIC>(p, pl, st);
        case 8: return launch_sparse<T, 64, 8, PAGED, MAGIC>(p, pl, st);
      }
      break;
    case 128:
      switch (pl.G_tile) {
        case 1: return launch_sparse<T, 128, 1, PAGED, MAGIC>(p, pl, st);
        case 2: return launch_sparse<T, 128, 2, PAGED, MAGIC>(p, pl, st);
        case 4: return launch_sparse<T, 128, 4, PAGED, MAGIC>(p, pl, st);
        case 8: return launch_sparse<T, 128, 8, PAGED, MAGIC>(p, pl, st);
      }
      break;
    case 256:
      switch (pl.G_tile) {
        case 1: return launch_sparse<T, 256, 1, PAGED, MAGIC>(p, pl, st);
        case 2: return launch_sparse<T, 256, 2, PAGED, MAGIC>(p, pl, st);
        case 4: return launch_sparse<T, 256, 4, PAGED, MAGIC>(p, pl, st);
      }
      break;
  }
  return set_error(AKT_ERR_UNSUPPORTED, "sparse decode: head_dim must be 64, 128 or 256");
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int check_heads(int B, int Hq, int Hkv, int D, int dtype, int max_nnz) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || max_nnz < 0) return set_error(AKT_ERR_INVALID, "sizes must be non-negative");
  if (Hq % Hkv != 0) return set_error(AKT_ERR_INVALID, "num_qo_heads must be a multiple of num_kv_heads");
  if (D != 64 && D != 128 && D != 256) return set_error(AKT_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
  if (dtype != AKT_FLOAT16 && dtype != AKT_BFLOAT16) return set_error(AKT_ERR_INVALID, "dtype");
  return AKT_OK;
}

void fill_common(SparseParams& p, const SparsePlan& pl, void* ws) {
  p.group = p.Hq / p.Hkv;
  p.g_tiles = p.group / pl.G_tile;
  p.units = p.Hkv * p.g_tiles;
  p.inline_plan = (int64_t)p.B * p.units <= kSThreads && pl.items > 0 ? 1 : 0;
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_lse = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.off_lse);
  p.unit_offset = reinterpret_cast<int*>(static_cast<char*>(ws) + pl.off_units);
}

int paged_entry(const akt_sparse_paged_args* a, void* ws, size_t ws_bytes, void* stream, bool magic,
                float* o_part = nullptr, float* lse_part = nullptr, const int32_t* csr_ptr = nullptr,
                int64_t num_inds = 0) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  int rc = check_heads(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype, a->max_nnz);
  if (rc) return rc;
  if (a->page_size <= 0) return set_error(AKT_ERR_INVALID, "page_size must be positive");
  if (magic && (!a->magicpig_k || !a->magicpig_l)) return set_error(AKT_ERR_INVALID, "MagicPIG needs K and L");
  if (a->q_stride_dim != 1 || a->kv_stride_dim != 1)
    return set_error(AKT_ERR_UNSUPPORTED, "sparse paged: unit dim stride required");
  if (!al16(a->q) || !al16(a->kv_cache) || (a->kv_stride_page % 8) || (a->kv_stride_kv % 8) ||
      (a->kv_stride_head % 8) || (a->kv_stride_token % 8) || (a->q_stride_batch % 8) || (a->q_stride_head % 8))
    return set_error(AKT_ERR_UNSUPPORTED, "sparse paged: 16-byte alignment required");
  if (a->batch == 0) return AKT_OK;
  SparsePlan pl = make_sparse_plan(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->max_nnz);
  if (!ws || ws_bytes < pl.ws_bytes) return set_error(AKT_ERR_WORKSPACE, "sparse paged: workspace too small");
  SparseParams p{};
  p.q = a->q; p.q_sb = a->q_stride_batch; p.q_sh = a->q_stride_head;
  p.k = a->kv_cache;
  p.v = static_cast<const char*>(a->kv_cache) + a->kv_stride_kv * 2;
  p.s0 = a->kv_stride_page; p.s_head = a->kv_stride_head; p.s_tok = a->kv_stride_token;
  p.indptr = a->kv_page_indptr; p.indices = a->kv_page_indices;
  p.num_pages = a->num_pages; p.num_page_entries = a->num_page_entries;
  p.ind = a->sparse_ind; p.ind_sb = a->ind_stride_batch; p.ind_sh = a->ind_stride_head; p.ind_sp = a->ind_stride_pos;
  p.nnz = a->sparse_nnz; p.nnz_sb = a->nnz_stride_batch; p.nnz_sh = a->nnz_stride_head;
  p.csr_ptr = csr_ptr; p.num_inds = num_inds;
  p.mp_k = a->magicpig_k; p.mp_l = a->magicpig_l; p.par_sb = a->param_stride_batch; p.par_sh = a->param_stride_head;
  p.out = a->out; p.o_sb = a->out_stride_batch; p.o_sh = a->out_stride_head; p.o_sd = a->out_stride_dim;
  p.B = a->batch; p.Hq = a->num_qo_heads; p.Hkv = a->num_kv_heads; p.L = 0; p.P = a->page_size;
  p.max_nnz = a->max_nnz;
  p.scale_log2 = a->softmax_scale * kLog2e;
  p.inv_sqrt_d = 1.0f / sqrtf((float)a->head_dim);
  fill_common(p, pl, ws);
  p.out_part_o = o_part;
  p.out_part_lse = lse_part;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (magic) {
    if (a->dtype == AKT_FLOAT16) return dispatch_sparse<__half, true, true>(p, pl, a->head_dim, st);
    return dispatch_sparse<__nv_bfloat16, true, true>(p, pl, a->head_dim, st);
  }
  if (a->dtype == AKT_FLOAT16) return dispatch_sparse<__half, true, false>(p, pl, a->head_dim, st);
  return dispatch_sparse<__nv_bfloat16, true, false>(p, pl, a->head_dim, st);
}

}  // namespace
}  // namespace akt

using namespace akt;

extern "C" {

size_t akt_sparse_dense_workspace_size(const akt_sparse_dense_args* a) {
  if (!a || check_heads(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype, a->max_nnz)) return 0;
  return make_sparse_plan(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->max_nnz).ws_bytes;
}

// descriptor of the peer-store exchange for the entry point running on this
// thread (set only for the duration of akt_sparse_dense_partial_peer)
static thread_local const akt_peer_exchange* g_peer = nullptr;
static thread_local bool g_peer_final = false;

static int sparse_dense_entry(const akt_sparse_dense_args* a, void* ws, size_t ws_bytes, void* stream,
                              float* o_part, float* lse_part, const int32_t* csr_ptr = nullptr,
                              int64_t num_inds = 0) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  int rc = check_heads(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype, a->max_nnz);
  if (rc) return rc;
  if (a->seq_len < 0) return set_error(AKT_ERR_INVALID, "seq_len < 0");
  if (a->q_stride_dim != 1 || a->k_stride_dim != 1 || a->v_stride_dim != 1)
    return set_error(AKT_ERR_UNSUPPORTED, "sparse dense: unit dim stride required");
  if (a->k_stride_batch != a->v_stride_batch || a->k_stride_head != a->v_stride_head ||
      a->k_stride_token != a->v_stride_token)
    return set_error(AKT_ERR_UNSUPPORTED, "sparse dense: K and V must share strides");
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || (a->k_stride_batch % 8) || (a->k_stride_head % 8) ||
      (a->k_stride_token % 8) || (a->q_stride_batch % 8) || (a->q_stride_head % 8))
    return set_error(AKT_ERR_UNSUPPORTED, "sparse dense: 16-byte alignment required");
  if (a->batch == 0) return AKT_OK;
  SparsePlan pl = make_sparse_plan(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->max_nnz);
  if (!ws || ws_bytes < pl.ws_bytes) return set_error(AKT_ERR_WORKSPACE, "sparse dense: workspace too small");
  SparseParams p{};
  p.q = a->q; p.q_sb = a->q_stride_batch; p.q_sh = a->q_stride_head;
  p.k = a->k; p.v = a->v;
  p.s0 = a->k_stride_batch; p.s_head = a->k_stride_head; p.s_tok = a->k_stride_token;
  p.ind = a->sparse_ind; p.ind_sb = a->ind_stride_batch; p.ind_sh = a->ind_stride_head; p.ind_sp = a->ind_stride_pos;
  p.nnz = a->sparse_nnz; p.nnz_sb = a->nnz_stride_batch; p.nnz_sh = a->nnz_stride_head;
  p.csr_ptr = csr_ptr; p.num_inds = num_inds;
  if (g_peer) {  // akt_sparse_dense_partial_peer / akt_sparse_dense_split_peer
    p.n_peers = g_peer->world;
    p.rank = g_peer->rank;
    p.epoch = g_peer->epoch;
    p.counter = g_peer->counter;
    for (int r = 0; r < g_peer->world; ++r) {
      p.peer_data[r] = g_peer->peer_data[r];
      p.peer_flags[r] = g_peer->peer_flags[r];
    }
    p.final_merge = g_peer_final ? 1 : 0;
    p.merge_counter = g_peer->merge_counter;
  }
  p.out = a->out; p.o_sb = a->out_stride_batch; p.o_sh = a->out_stride_head; p.o_sd = a->out_stride_dim;
  p.B = a->batch; p.Hq = a->num_qo_heads; p.Hkv = a->num_kv_heads; p.L = a->seq_len; p.P = 1;
  p.max_nnz = a->max_nnz;
  p.scale_log2 = a->softmax_scale * kLog2e;
  p.inv_sqrt_d = 1.0f / sqrtf((float)a->head_dim);
  fill_common(p, pl, ws);
  p.out_part_o = o_part;
  p.out_part_lse = lse_part;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == AKT_FLOAT16) return dispatch_sparse<__half, false, false>(p, pl, a->head_dim, st);
  return dispatch_sparse<__nv_bfloat16, false, false>(p, pl, a->head_dim, st);
}

int akt_sparse_dense(const akt_sparse_dense_args* a, void* ws, size_t ws_bytes, void* stream) {
  return sparse_dense_entry(a, ws, ws_bytes, stream, nullptr, nullptr);
}

int akt_sparse_dense_csr(const akt_sparse_dense_args* a, const int32_t* sparse_ptr, int64_t num_inds, void* ws,
                         size_t ws_bytes, void* stream) {
  if (!sparse_ptr || num_inds < 0) return set_error(AKT_ERR_INVALID, "CSR lists need sparse_ptr and num_inds >= 0");
  return sparse_dense_entry(a, ws, ws_bytes, stream, nullptr, nullptr, sparse_ptr, num_inds);
}

int akt_sparse_paged_csr(const akt_sparse_paged_args* a, const int32_t* sparse_ptr, int64_t num_inds, void* ws,
                         size_t ws_bytes, void* stream) {
  if (!sparse_ptr || num_inds < 0) return set_error(AKT_ERR_INVALID, "CSR lists need sparse_ptr and num_inds >= 0");
  return paged_entry(a, ws, ws_bytes, stream, false, nullptr, nullptr, sparse_ptr, num_inds);
}

int akt_magicpig_paged_csr(const akt_sparse_paged_args* a, const int32_t* sparse_ptr, int64_t num_inds, void* ws,
                           size_t ws_bytes, void* stream) {
  if (!sparse_ptr || num_inds < 0) return set_error(AKT_ERR_INVALID, "CSR lists need sparse_ptr and num_inds >= 0");
  return paged_entry(a, ws, ws_bytes, stream, true, nullptr, nullptr, sparse_ptr, num_inds);
}

int akt_sparse_dense_partial_peer(const akt_sparse_dense_args* a, const akt_peer_exchange* x, void* ws,
                                  size_t ws_bytes, void* stream) {
  if (!x || x->world < 1 || x->world > AKT_MAX_PEERS || x->rank < 0 || x->rank >= x->world || !x->counter ||
      x->epoch == 0)
    return set_error(AKT_ERR_INVALID, "peer exchange: bad descriptor");
  for (int r = 0; r < x->world; ++r)
    if (!x->peer_data[r] || !x->peer_flags[r]) return set_error(AKT_ERR_INVALID, "peer exchange: null peer pointer");
  g_peer = x;
  const int rc = sparse_dense_entry(a, ws, ws_bytes, stream, nullptr, nullptr);
  g_peer = nullptr;
  return rc;
}

int akt_sparse_dense_split_peer(const akt_sparse_dense_args* a, const akt_peer_exchange* x, void* ws,
                                size_t ws_bytes, void* stream) {
  if (!x || x->world < 1 || x->world > AKT_MAX_PEERS || x->rank < 0 || x->rank >= x->world || !x->counter ||
      !x->merge_counter || x->epoch == 0)
    return set_error(AKT_ERR_INVALID, "peer exchange: bad descriptor");
  for (int r = 0; r < x->world; ++r)
    if (!x->peer_data[r] || !x->peer_flags[r]) return set_error(AKT_ERR_INVALID, "peer exchange: null peer pointer");
  if (!a || !a->out) return set_error(AKT_ERR_INVALID, "split_peer: output required");
  // the merge grid waits on itself: it must be resident at once (one CTA per
  // (batch, unit), 256 threads, at most 64 registers each: four fit on every
  // SM; the launch also checks the occupancy the driver reports)
  if (a->num_kv_heads <= 0 || a->num_qo_heads % a->num_kv_heads) return set_error(AKT_ERR_INVALID, "heads");
  const int group = a->num_qo_heads / a->num_kv_heads;
  const int64_t units = (int64_t)a->batch * a->num_kv_heads * (group / sparse_group_tile(group, a->head_dim));
  if (units > (int64_t)sm_count() * 4)
    return set_error(AKT_ERR_UNSUPPORTED, "split_peer: too many (batch, unit) pairs for one resident merge grid");
  g_peer = x;
  g_peer_final = true;
  const int rc = sparse_dense_entry(a, ws, ws_bytes, stream, nullptr, nullptr);
  g_peer = nullptr;
  g_peer_final = false;
  return rc;
}

int akt_sparse_dense_partial(const akt_sparse_dense_args* a, float* o_part, float* lse_part, void* ws,
                             size_t ws_bytes, void* stream) {
  if (!o_part || !lse_part) return set_error(AKT_ERR_INVALID, "partial outputs required");
  return sparse_dense_entry(a, ws, ws_bytes, stream, o_part, lse_part);
}

int akt_sparse_paged_partial(const akt_sparse_paged_args* a, float* o_part, float* lse_part, void* ws,
                             size_t ws_bytes, void* stream) {
  if (!o_part || !lse_part) return set_error(AKT_ERR_INVALID, "partial outputs required");
  return paged_entry(a, ws, ws_bytes, stream, false, o_part, lse_part);
}

int akt_magicpig_paged_partial(const akt_sparse_paged_args* a, float* o_part, float* lse_part, void* ws,
                               size_t ws_bytes, void* stream) {
  if (!o_part || !lse_part) return set_error(AKT_ERR_INVALID, "partial outputs required");
  return paged_entry(a, ws, ws_bytes, stream, true, o_part, lse_part);
}

size_t akt_sparse_paged_workspace_size(const akt_sparse_paged_args* a) {
  if (!a || check_heads(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype, a->max_nnz)) return 0;
  return make_sparse_plan(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->max_nnz).ws_bytes;
}

int akt_sparse_paged(const akt_sparse_paged_args* a, void* ws, size_t ws_bytes, void* stream) {
  return paged_entry(a, ws, ws_bytes, stream, false);
}

size_t akt_magicpig_paged_workspace_size(const akt_sparse_paged_args* a) {
  return akt_sparse_paged_workspace_size(a);
}

int akt_magicpig_paged(const akt_sparse_paged_args* a, void* ws, size_t ws_bytes, void* stream) {
  return paged_entry(a, ws, ws_bytes, stream, true);
}

}  // extern "C"
