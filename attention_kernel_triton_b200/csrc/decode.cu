// Split-KV GQA decode for sm_100a: dense ("redundant") and paged var-len.
//
// Replaces the Triton kernels of decode_flash_attention_redundant.py:71-229
// and decode_flash_attention_redundant_var_len_paged.py:70-224.  Same math
// (one query row per qo head, softmax over every valid key, fp32
// accumulation; the reference's online-softmax recurrence is at DR:44-62 /
// DP:45-63), different machine mapping:
//
//  * GQA packing: one CTA owns (sequence, kv head, group of G qo heads,
//    chunk of tokens) and reads each K/V byte of its chunk once for all G
//    heads (the reference runs one program per qo head and re-reads K/V G
//    times, DP:124-127).
//  * Split-KV: a sequence's tokens are cut into chunks of C tokens; each chunk
//    is one CTA writing a partial (O normalised, log2-sum-exp) that the merge
//    kernel combines.  The reference scans a whole sequence in one program
//    (DP:168), with no LSE output.
//  * Staging: warp 0 is a producer that resolves page ids through the page
//    table and moves K and V tiles HBM->shared with 1-D bulk copies on the
//    TMA engine (cp.async.bulk + mbarrier complete_tx) into a ring of stages;
//    warps 1..4 consume tiles round-robin.  A tile never straddles a page.
//  * CUDA cores only (decode is HBM-bound): q.k with packed fp32x2 FMAs,
//    an 8-lane reduce-scatter that leaves each lane the score of one
//    (token, head), exp2 with the scale folded into q, P.V with fp32x2 FMAs.
#include "attn_core.cuh"
#include "attn_mma.cuh"
#include "tensor_map.h"
#include "common.cuh"
#include "profile.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <cstring>
#include <string>
#include <type_traits>

namespace akt {

__device__ unsigned int g_device_status = 0;



// status word of the prefill kernels (prefill.cu is whole-program device code)
cudaError_t prefill_status_read(unsigned int* v);
cudaError_t prefill_status_clear();

constexpr int kProducerWarps = 1;
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = 32 * (kProducerWarps + kConsumerWarps);
constexpr int kSubTile = kRowsPerSubTile;

struct DecodeParams {
  const void* q;
  int64_t q_sb, q_sh;  // q element strides (dim stride must be 1)
  // K/V addressing.  Dense: base of K / V, strides (batch, head, token).
  // Paged: k = pool, v = pool + stride_kv, strides (page, head, token).
  const void* k;
  const void* v;
  int64_t s0, s_head, s_tok;
  const int32_t* indptr;
  const int32_t* indices;
  const int32_t* last_len;
  int64_t num_pages;
  int64_t num_page_entries;
  void* out;
  int64_t o_sb, o_sh, o_sd;
  int B, Hq, Hkv;
  int L;  // dense sequence length
  int P;  // page size
  int group;          // Hq / Hkv
  int g_tiles;        // group / G_TILE
  int units;          // Hkv * g_tiles
  int tile_tokens;    // tokens per stage (divides P when paged)
  int chunk_tokens;   // multiple of tile_tokens
  int chunks_per_seq; // dense only
  int num_stages;
  float scale_log2;   // softmax_scale * log2(e)
  float* part_o;      // [items, G_TILE, D]
  float* part_lse;    // [items, G_TILE]   (log2 domain)
  // paged only: full-chunk offsets [B + 1], then the call's chunk count; with
  // tail_order, the sequences' partial last chunks come after every full one,
  // longest first: tail_seq[r] is the sequence of tail chunk r and
  // tail_rank[b] the rank of sequence b's tail (-1: none)
  int* chunk_offset;  // [B + 2]
  int* tail_seq;      // [B]
  int* tail_rank;     // [B]
  int tail_order;     // B <= 1024
  int max_chunks;     // paged: chunks the workspace holds per unit (the planner clamps to it)
  int direct_out;     // every unit has one chunk: write O directly
};

// ---------------------------------------------------------------------------
// planner: per-sequence chunk counts -> exclusive prefix (one CTA)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int paged_seq_len(const DecodeParams& p, int b) {
  int s = p.indptr[b], e = p.indptr[b + 1];
  int np = e - s;
  if (np <= 0) return 0;
  int last = p.last_len[b];
  last = last < 0 ? 0 : (last > p.P ? p.P : last);
  return (np - 1) * p.P + last;
}

// Chunk order.  The split-KV CTAs start in chunk order, and a CTA's time
// follows its tokens, so a sequence's partial last chunk is a short job.  With
// tail_order (up to 1024 sequences, one thread each) every sequence's full
// chunks come first, in sequence order, and the partial last chunks after all
// of them, longest first, so the last wave of CTAs holds the short jobs
// (list scheduling of cfg3's chunks on 3 x 148 slots: 5.4 % above the ideal
// makespan in plain order, 2.5 % in this one).  Larger batches keep the plain
// order (every chunk of a sequence in place).
//
// Chunk counts are clamped to p.max_chunks, the count the workspace was sized
// for (num_page_entries * P / chunk_tokens + B, which a well-formed indptr never
// exceeds: its ranges are disjoint and inside the index array).  An indptr whose
// ranges overlap can ask for more; its excess chunks are dropped and recorded as
// kStatusBadIndptr, so neither the split-KV kernel nor the merge ever reads or
// writes past the workspace.
__global__ void __launch_bounds__(1024) paged_plan_kernel(DecodeParams p) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  __shared__ int rem_s[1024];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < p.B; base += 1024) {
    int b = base + threadIdx.x;
    int n = 0, rem = 0;
    if (b < p.B) {
      int s = p.indptr[b], e = p.indptr[b + 1];
      if (e < s || s < 0 || e > p.num_page_entries) {
        record_status(kStatusBadIndptr);
      } else {
        const int len = paged_seq_len(p, b);
        // at most max_chunks + 1 per sequence, so the sums below cannot overflow
        n = min(p.tail_order ? len / p.chunk_tokens : cdiv(len, p.chunk_tokens), p.max_chunks + 1);
        rem = p.tail_order ? len - (len / p.chunk_tokens) * p.chunk_tokens : 0;
      }
      p.tail_rank[b] = -1;
    }
    if (p.tail_order) rem_s[threadIdx.x] = b < p.B ? rem : 0;
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? warp_sums[warp - 1] : 0);  // inclusive, within this block
    if (b < p.B) p.chunk_offset[b] = min(carry + incl - n, p.max_chunks);
    __syncthreads();
    if (threadIdx.x == 1023) carry = min(carry + incl, p.max_chunks + 1);  // block total (n == 0 past the end)
    __syncthreads();
    if (p.tail_order && b < p.B && rem > 0) {  // one block: all sequences are in rem_s
      int rank = 0;
      for (int o = 0; o < p.B; ++o) {
        const int ro = rem_s[o];
        rank += (ro > rem || (ro == rem && o < b)) ? 1 : 0;
      }
      const int full = min(carry, p.max_chunks);
      if (full + rank < p.max_chunks) {
        p.tail_rank[b] = rank;
        p.tail_seq[rank] = b;
      } else {
        record_status(kStatusBadIndptr);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (carry > p.max_chunks) record_status(kStatusBadIndptr);
    const int full = min(carry, p.max_chunks);
    int tails = 0;
    if (p.tail_order)
      for (int o = 0; o < p.B; ++o) tails += (rem_s[o] > 0 && p.tail_rank[o] >= 0) ? 1 : 0;
    p.chunk_offset[p.B] = full;
    p.chunk_offset[p.B + 1] = full + tails;
  }
}

// ---------------------------------------------------------------------------
// main split-KV kernel
// ---------------------------------------------------------------------------
// The consumer warps' combined state -> the item's partial (O normalised,
// log2-sum-exp), or the output row when the unit has one chunk.
template <typename T, int D, int G>
__device__ __forceinline__ void write_item(const DecodeParams& p, int item, int b, int head0, const float* comb_m,
                                           const float* comb_l, const float* comb_o, int ctid) {
  using E = Elem<T>;
  T* out = static_cast<T*>(p.out);
  for (int e = ctid; e < G * D; e += kConsumerWarps * 32) {
    const int h = e / D, d = e - h * D;
    float lse2;
    const float val = combine_warps<kConsumerWarps, G, D>(comb_m, comb_l, comb_o, h, d, lse2);
    if (p.direct_out) {
      out[(int64_t)b * p.o_sb + (int64_t)(head0 + h) * p.o_sh + (int64_t)d * p.o_sd] = E::from_float(val);
    } else {
      p.part_o[((int64_t)item * G + h) * D + d] = val;
      if (d == 0) p.part_lse[(int64_t)item * G + h] = lse2;
    }
  }
}

// Work item (blockIdx.x) -> sequence b, chunk c of it, the sequence's length.
// Returns false when the item has no chunk (paged bound past the call's count).
// seq_s: three ints of shared scratch (paged calls).
template <bool PAGED>
__device__ __forceinline__ bool resolve_item(const DecodeParams& p, int cg, int& b, int& c, int& seq_len,
                                             int* seq_s) {
  if (PAGED) {
    grid_dep_wait();  // chunk offsets come from the planner kernel
    const int total = p.chunk_offset[p.B + 1], full = p.chunk_offset[p.B];
    if (cg >= total) return false;
    if (cg >= full) {  // a partial last chunk, after every full one
      b = p.tail_seq[cg - full];
      seq_len = paged_seq_len(p, b);
      c = seq_len / p.chunk_tokens;
    } else if (p.B <= kDecodeThreads) {
      // one thread per sequence, all loads in one round: the sequence whose
      // chunk range holds cg (exactly one; empty ranges never match) publishes
      // itself, the chunk index and its length (a binary search is a chain of
      // dependent loads ahead of the CTA's first copy)
      const int t = threadIdx.x;
      if (t < p.B) {
        const int a = p.chunk_offset[t], z = p.chunk_offset[t + 1];
        const int len = paged_seq_len(p, t);
        if (a <= cg && cg < z) {
          seq_s[0] = t;
          seq_s[1] = cg - a;
          seq_s[2] = len;
        }
      }
      __syncthreads();
      b = seq_s[0];
      c = seq_s[1];
      seq_len = seq_s[2];
    } else {
      int lo = 0, hi = p.B - 1;  // largest b with chunk_offset[b] <= cg
      while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (p.chunk_offset[mid] <= cg) lo = mid; else hi = mid - 1;
      }
      b = lo;
      c = cg - p.chunk_offset[b];
      seq_len = paged_seq_len(p, b);
    }
  } else {
    b = cg / p.chunks_per_seq;
    c = cg - b * p.chunks_per_seq;
    seq_len = p.L;
  }
  return true;
}

template <typename T, int D, int G, bool PAGED>
__global__ void __launch_bounds__(kDecodeThreads, (G * D > 512) ? 2 : 3) decode_splitkv_kernel(const DecodeParams p) {
  static_assert(D % 64 == 0 && D <= 256, "head_dim");
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "group tile");
  using E = Elem<T>;

  extern __shared__ __align__(128) unsigned char smem[];
  const int NS = p.num_stages;
  const int TT = p.tile_tokens;
  const int stage_elems = TT * D;
  T* kv_s = reinterpret_cast<T*>(smem);  // [NS][2][TT][D]
  float* comb = reinterpret_cast<float*>(smem + (size_t)NS * 2 * stage_elems * sizeof(T));
  float* comb_m = comb;                               // [NW][G]
  float* comb_l = comb_m + kConsumerWarps * G;        // [NW][G]
  float* comb_o = comb_l + kConsumerWarps * G;        // [NW][G][D]
  float* p_s = comb_o + kConsumerWarps * G * D;       // [NW][kSubTile][G]
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kConsumerWarps * kSubTile * G);
  uint64_t* full = bars;        // [NS]
  uint64_t* empty = bars + NS;  // [NS]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work item -> (sequence, unit, token range)
  const int item = blockIdx.x;
  const int cg = item / p.units;
  const int unit = item - cg * p.units;
  int b, c, seq_len;
  __shared__ int seq_s[3];
  if (!resolve_item<PAGED>(p, cg, b, c, seq_len, seq_s)) return;
  const int tok_begin = c * p.chunk_tokens;
  const int tok_end = min(seq_len, tok_begin + p.chunk_tokens);
  const int n_tiles = cdiv(tok_end - tok_begin, TT);
  const int kvh = unit / p.g_tiles;
  const int head0 = kvh * p.group + (unit - kvh * p.g_tiles) * G;

  if (NS % kConsumerWarps != 0) {  // host guarantees this; never run a mis-phased ring
    if (threadIdx.x == 0) record_status(kStatusWaitTimeout);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp < kProducerWarps) {
    // ======================= producer =======================
    const uint64_t pol = l2_policy_evict_first();
    const uint32_t row_bytes = D * sizeof(T);
    const T* kbase = static_cast<const T*>(p.k);
    const T* vbase = static_cast<const T*>(p.v);
    int page_base = 0, npages = 0, batch_lo = -1, my_pid = -1, issued = 0;
    if (PAGED) {
      page_base = p.indptr[b];
      npages = p.indptr[b + 1] - page_base;
    }
    for (int t = 0; t < n_tiles; ++t) {
      const int slot = t % NS;
      const uint32_t phase = (uint32_t)(t / NS) & 1u;
      const int tok = tok_begin + t * TT;
      const int n = min(TT, tok_end - tok);
      int64_t off;
      bool ok_addr = true;
      if (PAGED) {
        const int pl = tok / p.P;
        if (batch_lo < 0 || pl >= batch_lo + 32) {
          batch_lo = pl;
          const int j = batch_lo + lane;
          my_pid = (j < npages) ? __ldg(p.indices + page_base + j) : -1;
        }
        const int pid = __shfl_sync(0xffffffffu, my_pid, pl - batch_lo);
        if (pid < 0 || (int64_t)pid >= p.num_pages) {
          ok_addr = false;
          off = 0;
        } else {
          off = (int64_t)pid * p.s0 + (int64_t)kvh * p.s_head + (int64_t)(tok - pl * p.P) * p.s_tok;
        }
      } else {
        off = (int64_t)b * p.s0 + (int64_t)kvh * p.s_head + (int64_t)tok * p.s_tok;
      }
      bool ok = true;
      if (t >= NS && lane == 0) ok = mbar_wait(&empty[slot], phase ^ 1u);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      issued = t + 1;
      if (lane == 0) {
        T* dst = kv_s + (size_t)slot * 2 * stage_elems;
        if (ok_addr) {
          const uint32_t bytes = (uint32_t)n * row_bytes;
          mbar_arrive_expect_tx(&full[slot], 2u * bytes);
          bulk_g2s(dst, kbase + off, bytes, &full[slot], pol);
          bulk_g2s(dst + stage_elems, vbase + off, bytes, &full[slot], pol);
        } else {
          record_status(kStatusBadPage);
          mbar_arrive(&full[slot]);
        }
      }
      __syncwarp();
    }
    // Do not exit while bulk copies into this CTA's shared memory are in
    // flight: wait (bounded) for the full barrier of every issued tile that
    // no consumer has waited on yet (consumers wait on all of them on the
    // normal path, so this returns at once there).
    if (lane == 0) {
      for (int t = max(0, issued - NS); t < issued; ++t) mbar_wait(&full[t % NS], (uint32_t)(t / NS) & 1u);
    }
    return;
  }

  // ========================= consumers =========================
  const int cw = warp - kProducerWarps;
  WarpAttn<T, D, G, false> wa;
  wa.init(lane);
  wa.load_q(static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)head0 * p.q_sh, p.q_sh, p.scale_log2);
  float* pw = p_s + cw * kSubTile * G;
  bool alive = true;
  const ScaledDotScore score;

  for (int t = cw; t < n_tiles; t += kConsumerWarps) {
    const int slot = t % NS;
    if (!mbar_wait(&full[slot], (uint32_t)(t / NS) & 1u)) { alive = false; break; }
    const int n = min(TT, tok_end - (tok_begin + t * TT));
    const T* Ks = kv_s + (size_t)slot * 2 * stage_elems;
    const T* Vs = Ks + stage_elems;
    for (int sub = 0; sub < n; sub += kSubTile)
      wa.step(Ks, Vs, sub, min(kSubTile, n - sub), TT - 1, 0xffffffffu, pw, score);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // ---- combine the consumer warps' states
  wa.stash(comb_m, comb_l, comb_o, cw, alive);
  named_bar_sync(1, kConsumerWarps * 32);
  write_item<T, D, G>(p, item, b, head0, comb_m, comb_l, comb_o, threadIdx.x - 32 * kProducerWarps);
}

// ---------------------------------------------------------------------------
// Split-KV decode on the tensor cores: the same work items, chunk order,
// producer ring and combine as decode_splitkv_kernel, with
//  * the producer loading each tile through two 4-D tensor maps (K and V:
//    [D, tokens, kv heads, pages or sequences]) with a 128-byte swizzle, one
//    64-column box per half of D, so the consumers' ldmatrix reads are free of
//    bank conflicts (the 1-D bulk copies land rows 256 bytes apart, which puts
//    the 8 rows an ldmatrix phase reads in the same banks);
//  * consumer warps running WarpMma (16 keys per step, two m16n8k16 products)
//    instead of the CUDA-core warp core.
// A tile is TT keys (a multiple of 16).  The box always moves TT rows: rows past
// the sequence end inside a page are the pool's own bytes, so a consumer
// zeroes those V rows before its step (a masked key's p is 0, and 0 * NaN is
// NaN on the tensor cores too); dense rows past L are filled with zeros by the
// tensor-map load.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Paged calls below D=256 run four CTAs per SM (at most 102 registers, a 32 KB
// stage ring each); the others three (64 KB rings; at D=256 the consumers
// need more registers).  See the stage budget in make_plan.
template <int D, bool PAGED>
constexpr int mma_ctas_per_sm() { return (PAGED && D < 256) ? 4 : 3; }

template <typename T, int D, int G, bool PAGED>
__global__ void __launch_bounds__(kDecodeThreads, mma_ctas_per_sm<D, PAGED>())
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const DecodeParams p) {
  static_assert(D % 64 == 0 && D <= 256, "head_dim");
  // Stages on 1024-byte boundaries: the tensor-map loads' 128-byte swizzle
  // repeats every 1024 bytes.  The kernel declares no static shared memory,
  // so the dynamic region starts the CTA's window; the check below reads its
  // address through an opaque move (the declared alignment would let the
  // compiler drop a plain test) and stops the CTA before any load if it is off.
  extern __shared__ __align__(1024) unsigned char smem_tc[];
  unsigned char* smem = smem_tc;
  uint32_t smem_base;
  asm volatile("mov.b32 %0, %1;" : "=r"(smem_base) : "r"(smem_u32(smem_tc)));
  const int NS = p.num_stages;
  const int TT = p.tile_tokens;
  const int stage_elems = TT * D;  // one matrix of a stage: [D / 64][TT][64]
  const uint32_t mat_bytes = (uint32_t)stage_elems * sizeof(T);
  const uint32_t half_bytes = (uint32_t)TT * 128u;
  T* kv_s = reinterpret_cast<T*>(smem);  // [NS][2][D / 64][TT][64]
  float* comb_m = reinterpret_cast<float*>(smem + (size_t)NS * 2 * mat_bytes);  // [NW][G]
  float* comb_l = comb_m + kConsumerWarps * G;                                 // [NW][G]
  float* comb_o = comb_l + kConsumerWarps * G;                                 // [NW][G][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(comb_o + kConsumerWarps * G * D);  // [NS]
  uint64_t* empty = full + NS;                                                    // [NS]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int item = blockIdx.x;
  const int cg = item / p.units;
  const int unit = item - cg * p.units;
  int b, c, seq_len;
  // the lookup's scratch: the first ints of comb_m (written only at the end)
  if (!resolve_item<PAGED>(p, cg, b, c, seq_len, reinterpret_cast<int*>(comb_m))) return;
  const int tok_begin = c * p.chunk_tokens;
  const int tok_end = min(seq_len, tok_begin + p.chunk_tokens);
  const int n_tiles = cdiv(tok_end - tok_begin, TT);
  const int kvh = unit / p.g_tiles;
  const int head0 = kvh * p.group + (unit - kvh * p.g_tiles) * G;

  if (NS % kConsumerWarps != 0 || (TT & 15) != 0 || (smem_base & 1023u) != 0) {  // host guarantees these
    if (threadIdx.x == 0) record_status(kStatusWaitTimeout);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp < kProducerWarps) {
    // ======================= producer =======================
    const uint64_t pol = l2_policy_evict_first();
    int page_base = 0, npages = 0, batch_lo = -1, my_pid = -1, issued = 0;
    if (PAGED) {
      page_base = p.indptr[b];
      npages = p.indptr[b + 1] - page_base;
    }
    for (int t = 0; t < n_tiles; ++t) {
      const int slot = t % NS;
      const uint32_t phase = (uint32_t)(t / NS) & 1u;
      const int tok = tok_begin + t * TT;
      int y, w;  // token coordinate inside the page / sequence; page id / sequence
      bool ok_addr = true;
      if (PAGED) {
        const int pl = tok / p.P;
        if (batch_lo < 0 || pl >= batch_lo + 32) {
          batch_lo = pl;
          const int j = batch_lo + lane;
          my_pid = (j < npages) ? __ldg(p.indices + page_base + j) : -1;
        }
        const int pid = __shfl_sync(0xffffffffu, my_pid, pl - batch_lo);
        ok_addr = pid >= 0 && (int64_t)pid < p.num_pages;
        y = tok - pl * p.P;
        w = pid;
      } else {
        y = tok;
        w = b;
      }
      bool ok = true;
      if (t >= NS && lane == 0) ok = mbar_wait(&empty[slot], phase ^ 1u);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      issued = t + 1;
      if (lane == 0) {
        T* dst = kv_s + (size_t)slot * 2 * stage_elems;
        if (ok_addr) {
          mbar_arrive_expect_tx(&full[slot], 2u * mat_bytes);
#pragma unroll
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d_hint(dst + hh * TT * 64, &tmK, hh * 64, y, kvh, w, &full[slot], pol);
            tma_load_4d_hint(dst + stage_elems + hh * TT * 64, &tmV, hh * 64, y, kvh, w, &full[slot], pol);
          }
        } else {
          record_status(kStatusBadPage);
          mbar_arrive(&full[slot]);
        }
      }
      __syncwarp();
    }
    // no exit while tensor-map loads into this CTA's shared memory are in
    // flight (bounded waits; returns at once on the normal path)
    if (lane == 0) {
      for (int t = max(0, issued - NS); t < issued; ++t) mbar_wait(&full[t % NS], (uint32_t)(t / NS) & 1u);
    }
    return;
  }

  // ========================= consumers =========================
  const int cw = warp - kProducerWarps;
  WarpMma<T, D, G> wm;
  wm.init(lane);
  wm.load_q(static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)head0 * p.q_sh, p.q_sh);
  bool alive = true;
  for (int t = cw; t < n_tiles; t += kConsumerWarps) {
    const int slot = t % NS;
    if (!mbar_wait(&full[slot], (uint32_t)(t / NS) & 1u)) { alive = false; break; }
    const int n = min(TT, tok_end - (tok_begin + t * TT));
    T* ks = kv_s + (size_t)slot * 2 * stage_elems;
    const uint32_t kb = smem_u32(ks);
    bool zeroed = false;
    if (PAGED && n < TT) {
      // rows n..TT-1 of V: whole 128-byte rows of every half
      unsigned char* vg = reinterpret_cast<unsigned char*>(ks + stage_elems);
      const int per_half = (TT - n) * 8;
      for (int e = lane; e < per_half * (D / 64); e += 32) {
        const int hh = e / per_half, r = e - hh * per_half;
        *reinterpret_cast<uint4*>(vg + hh * half_bytes + (n + (r >> 3)) * 128 + (r & 7) * 16) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
      zeroed = true;
    }
    for (int sub = 0; sub < n; sub += 16)
      wm.step(kb, kb + mat_bytes, half_bytes, sub, min(16, n - sub), p.scale_log2);
    __syncwarp();
    if (zeroed) fence_proxy_async_smem();  // generic writes before the next tensor-map load of the slot
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  wm.stash(comb_m, comb_l, comb_o, cw, alive);
  named_bar_sync(1, kConsumerWarps * 32);
  write_item<T, D, G>(p, item, b, head0, comb_m, comb_l, comb_o, threadIdx.x - 32 * kProducerWarps);
}

// ---------------------------------------------------------------------------
// merge of split-KV partials: O = sum_j 2^{lse_j - M} O_j / sum_j 2^{lse_j - M}
// One CTA per (sequence, unit).  Per head, one warp takes the max and the sum
// of 2^(lse_j - M) over the chunks (lanes striding the chunks).  Then the
// threads form blockDim / (G * D / 4) groups; in each group a thread
// accumulates four consecutive dims of one head over every groups-th chunk
// (one 16-byte load per chunk, unrolled so several loads are in flight), and
// the groups' sums are added in shared memory.  The host launches 1024
// threads when the chunk lists are long (16 chunks or more per pair; a
// single long sequence has ~50), and 256 otherwise.
// ---------------------------------------------------------------------------
template <typename T, int D, int G, bool PAGED>
__global__ void __launch_bounds__(1024) decode_merge_kernel(const DecodeParams p) {
  using E = Elem<T>;
  grid_dep_wait();  // partials (and chunk offsets) of the previous kernels
  const int b = blockIdx.x / p.units;
  const int unit = blockIdx.x - b * p.units;
  // chunks c0 .. c1-1 and, paged with a tail chunk, one more: item `tail`
  int c0, c1, tail = -1;
  if (PAGED) {
    c0 = p.chunk_offset[b];
    c1 = p.chunk_offset[b + 1];
    const int r = p.tail_rank[b];
    if (r >= 0) tail = p.chunk_offset[p.B] + r;
  } else {
    c0 = b * p.chunks_per_seq;
    c1 = c0 + p.chunks_per_seq;
  }
  const int nc = c1 - c0 + (tail >= 0 ? 1 : 0);
  auto chunk = [&](int k) { return k < c1 - c0 ? c0 + k : tail; };
  const int kvh = unit / p.g_tiles;
  const int head0 = kvh * p.group + (unit - kvh * p.g_tiles) * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float head_m[G], head_inv[G];
  constexpr int NE = G * D / 4;  // four-dim elements of the unit's output
  static_assert(NE <= 256, "elements per unit");
  __shared__ float4 red[1024 - NE];  // sums of groups 1.. (blockDim <= 1024)
  for (int h = warp; h < G; h += (int)(blockDim.x >> 5)) {
    float m = -INFINITY;
    for (int k = lane; k < nc; k += 32) m = fmaxf(m, p.part_lse[((int64_t)chunk(k) * p.units + unit) * G + h]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float den = 0.f;
    if (m != -INFINITY)
      for (int k = lane; k < nc; k += 32)
        den += fast_exp2(p.part_lse[((int64_t)chunk(k) * p.units + unit) * G + h] - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (lane == 0) {
      head_m[h] = m;
      head_inv[h] = den > 0.f ? 1.f / den : 0.f;
    }
  }
  __syncthreads();
  const int groups = max(1, (int)blockDim.x / NE);
  const int gi = threadIdx.x / NE, e4 = threadIdx.x - gi * NE;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
  const int h = (4 * e4) / D, d = 4 * e4 - h * D;
  if (gi < groups) {
    const float M = head_m[h];
    if (M != -INFINITY) {
#pragma unroll 8
      for (int k = gi; k < nc; k += groups) {
        const int64_t it = (int64_t)chunk(k) * p.units + unit;
        const float w = fast_exp2(p.part_lse[it * G + h] - M);
        const float4 o = *reinterpret_cast<const float4*>(p.part_o + (it * G + h) * D + d);
        num.x += w * o.x;
        num.y += w * o.y;
        num.z += w * o.z;
        num.w += w * o.w;
      }
    }
    if (gi > 0) red[(gi - 1) * NE + e4] = num;
  }
  if (groups > 1) __syncthreads();
  if (gi == 0) {
    for (int g2 = 1; g2 < groups; ++g2) {
      const float4 o = red[(g2 - 1) * NE + e4];
      num.x += o.x;
      num.y += o.y;
      num.z += o.z;
      num.w += o.w;
    }
    const float inv = head_inv[h];
    T* out = static_cast<T*>(p.out);
    T* orow = out + (int64_t)b * p.o_sb + (int64_t)(head0 + h) * p.o_sh;
    orow[(int64_t)d * p.o_sd] = E::from_float(num.x * inv);
    orow[(int64_t)(d + 1) * p.o_sd] = E::from_float(num.y * inv);
    orow[(int64_t)(d + 2) * p.o_sd] = E::from_float(num.z * inv);
    orow[(int64_t)(d + 3) * p.o_sd] = E::from_float(num.w * inv);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  static thread_local int cached_dev = -1, cached = 0;
  if (dev != cached_dev) {
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
    if (cached <= 0) cached = 148;
    cached_dev = dev;
  }
  return cached;
}

namespace {

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Plan {
  int G_tile, tile_tokens, chunk_tokens, num_stages;
  int64_t items;  // upper bound (paged) or exact (dense)
  int chunks_per_seq;
  size_t smem;     // CUDA-core kernel
  size_t smem_tc;  // tensor-core kernel
  bool tc;         // tiles fit the tensor-core kernel (a multiple of 16 keys)
  size_t ws_bytes;
  size_t off_lse, off_chunk;
  bool direct;
};

// Item count and workspace layout of a plan whose chunk length is set:
// partial O [items][G][D] fp32, partial log2-sum-exp [items][G] (when there
// is more than one chunk per unit) and, paged, the chunk order: offsets and
// counts [B + 2], tail chunks' sequences [B] and sequences' tail ranks [B].  Paged item counts are the
// bound num_page_entries * P / chunk_tokens + B chunks per unit.
void layout_workspace(Plan& pl, bool paged, int B, int units, int D, int L, int P, int64_t num_page_entries) {
  if (paged) {
    const int64_t chunks = num_page_entries * (int64_t)P / pl.chunk_tokens + B;
    pl.items = chunks * units;
    pl.chunks_per_seq = 0;
    pl.direct = false;
  } else {
    pl.chunks_per_seq = std::max(1, cdiv(L, pl.chunk_tokens));
    pl.items = (int64_t)B * pl.chunks_per_seq * units;
    pl.direct = pl.chunks_per_seq == 1;
  }
  size_t ws = 0;
  if (!pl.direct) {
    ws = align_up((size_t)pl.items * pl.G_tile * D * sizeof(float), 256);
    pl.off_lse = ws;
    ws += align_up((size_t)pl.items * pl.G_tile * sizeof(float), 256);
  }
  pl.off_chunk = ws;
  if (paged) ws += align_up((size_t)(3 * B + 2) * sizeof(int), 256);
  pl.ws_bytes = ws;
}

// Tuning knobs, read once per thread: AKT_DECODE_STAGE_KB (shared-memory
// budget of the K/V stage ring per CTA, default 64; 32 for paged tensor-core
// calls below D=256), AKT_DECODE_CHUNK_TILES (upper bound on tiles per
// split-KV chunk, default 128; dense inputs count 16 KB tiles, two of their
// 8 KB ones) and AKT_DECODE_ITEMS_PER_SM (work items aimed at per SM, default
// 3: about one wave at three CTAs per SM; large inputs hit the chunk bound
// instead).
int env_int(const char* name, int dflt) {
  // the environment's value is cached (0: unset); the default is the call's
  static thread_local int cache[3] = {-1, -1, -1};
  const char k = name[11];
  int* slot = &cache[k == 'S' ? 0 : k == 'C' ? 1 : 2];
  if (*slot < 0) {
    const char* v = getenv(name);
    const int x = v ? atoi(v) : 0;
    *slot = x > 0 ? x : 0;
  }
  return *slot > 0 ? *slot : dflt;
}

// AKT_DECODE_TENSOR_CORES=0 selects the CUDA-core split-KV kernel for every
// call (default: the tensor-core kernel wherever the tiles fit it).
bool use_tensor_cores() {
  static const bool on = [] {
    const char* v = getenv("AKT_DECODE_TENSOR_CORES");
    return !(v && v[0] == '0');
  }();
  return on;
}

int pick_group_tile(int group, int D) {
  const int cap = D >= 256 ? 4 : 8;
  for (int g = cap; g >= 2; g >>= 1)
    if (group % g == 0) return g;
  return 1;
}

int largest_divisor_le(int n, int cap) {
  for (int d = std::min(n, cap); d >= 1; --d)
    if (n % d == 0) return d;
  return 1;
}


Plan make_plan(bool paged, int B, int Hq, int Hkv, int D, int L, int P, int64_t num_page_entries,
               size_t elem_size) {
  Plan pl{};
  const int group = Hq / Hkv;
  pl.G_tile = pick_group_tile(group, D);
  const int units = Hkv * (group / pl.G_tile);
  const int tcap = (int)(4096 / D);  // stage of K+V tiles <= 16 KB
  // Dense tiles are half that (8 KB stages, at least one 16-row step): the
  // 64 KB ring then holds two stages per consumer warp, so a warp's next tile
  // loads while it works on the current one.  With few CTAs per SM (short
  // inputs) nothing else hides that load: 4 % faster on 8 x 1024 tokens at
  // D=64, 5 % on 4096 tokens at D=128.  (Paged tiles divide the page: 16
  // tokens at P=16, already two stages per warp.)
  const int dense_split = std::max(1, tcap / std::max(kSubTile, tcap / 2));
  pl.tile_tokens = paged ? largest_divisor_le(P, tcap) : tcap / dense_split;
  // The tensor-core kernel takes tiles of a multiple of 16 keys: the largest
  // such divisor of the page (pages of a multiple of 16 keys; others keep the
  // CUDA-core kernel).  Dense tiles are 16 or 32 keys already.
  if (paged && P % 16 == 0) {
    for (int d = (tcap / 16) * 16; d >= 16; d -= 16)
      if (P % d == 0) { pl.tile_tokens = d; break; }
  }
  pl.tc = pl.tile_tokens % 16 == 0 && use_tensor_cores();
  const size_t stage_bytes = (size_t)2 * pl.tile_tokens * D * elem_size;
  // Consumer warp w takes tiles w, w+NW, ...; with NS a multiple of NW every
  // slot has one fixed consumer, so each mbarrier is waited phase by phase
  // (a parity wait is only unambiguous for the current or previous phase).
  // Paged tensor-core calls below D=256: 32 KB rings (one stage per consumer
  // warp) so that four CTAs fit per SM.  cfg3: kernel 764 -> 690 us (3 CTAs with
  // 64 KB rings against 4 with 32 KB).  Dense calls keep 64 KB rings with three
  // CTAs: at L=128K the 4-CTA form took 84.3 us against 81.1.
  const bool four_per_sm = paged && pl.tc && D < 256;
  const size_t fit = (size_t)env_int("AKT_DECODE_STAGE_KB", four_per_sm ? 32 : 64) * 1024 / stage_bytes;
  pl.num_stages = (int)std::max<size_t>(kConsumerWarps, std::min<size_t>(16, fit / kConsumerWarps * kConsumerWarps));
  // estimated tiles over all units -> chunk size: aim for about one wave of
  // CTAs (3 per SM), but no more than AKT_DECODE_CHUNK_TILES tiles per chunk
  int64_t tiles_per_unit;
  if (paged) {
    tiles_per_unit = num_page_entries * (int64_t)(P / pl.tile_tokens);
  } else {
    tiles_per_unit = (int64_t)B * cdiv(L, pl.tile_tokens);
  }
  const int64_t total_tiles = std::max<int64_t>(1, tiles_per_unit * units);
  // work items aimed at per SM: three (one wave at three CTAs per SM).  With
  // 8 KB dense stages this is also the best for dense inputs with many
  // (sequence, unit) pairs (8 x 1024 tokens at D=64: 16.9 us against 18.4 at two)
  // (three also with four CTAs per SM: eight cfg3-like sequences took 90.9 us
  // at four, 81.9 at three; 16 and 32 sequences and cfg3 the same either way)
  const int ips = env_int("AKT_DECODE_ITEMS_PER_SM", 3);
  const int64_t target = (int64_t)sm_count() * ips;
  int64_t ct = (total_tiles + target - 1) / target;
  if (paged) {
    // One wave of CTAs when the chunks fit the bound: the chunk length that
    // fills `target` slots.  Otherwise bound-length chunks, unless they make
    // between 1.25 and 4 waves: then the last wave runs part-empty, and chunks
    // short enough for four waves are faster (one GPU's share of cfg3 split by
    // kv head: one head 169 -> 155 us, two heads 271 -> 261 us).  Just over one
    // wave stays (8 cfg3-like sequences: 105 us at 120-tile chunks, 118 us
    // with four waves: the few CTAs left at the end run faster alone).
    const int64_t one_wave = ct;
    const int64_t max_ct_paged = env_int("AKT_DECODE_CHUNK_TILES", 128);
    const double waves = (double)(total_tiles / max_ct_paged + (int64_t)B * units) / (double)target;
    if (one_wave <= max_ct_paged)
      ct = one_wave;
    else if (waves >= 1.25 && waves < 4.0)
      ct = std::max<int64_t>(16, std::min<int64_t>(max_ct_paged, total_tiles / (4 * target)));
    else
      ct = max_ct_paged;
  } else {
    // dense: chunks are cut per (sequence, unit), so size them from the chunks
    // each one may take (the rounding of a total-based size can add a wave)
    const int64_t seq_tiles = std::max<int64_t>(1, cdiv(L, pl.tile_tokens));
    const int64_t per_seq = std::max<int64_t>(1, target / std::max<int64_t>(1, (int64_t)B * units));
    ct = (seq_tiles + per_seq - 1) / per_seq;
  }
  // the chunk bound counts 16 KB tiles: dense chunks keep their length in tokens
  const int64_t max_ct = (int64_t)env_int("AKT_DECODE_CHUNK_TILES", 128) * (paged ? 1 : dense_split);
  ct = std::max<int64_t>(1, std::min<int64_t>(max_ct, ct));
  pl.chunk_tokens = (int)(ct * pl.tile_tokens);
  pl.smem = (size_t)pl.num_stages * stage_bytes +
            sizeof(float) * ((size_t)kConsumerWarps * pl.G_tile * (2 + D) + (size_t)kConsumerWarps * kSubTile * pl.G_tile) +
            sizeof(uint64_t) * 2 * pl.num_stages;
  pl.smem_tc = (size_t)pl.num_stages * stage_bytes + sizeof(float) * (size_t)kConsumerWarps * pl.G_tile * (2 + D) +
               sizeof(uint64_t) * 2 * pl.num_stages;
  layout_workspace(pl, paged, B, units, D, L, P, num_page_entries);
  return pl;
}

// K and V tensor maps of the tensor-core kernel: [D, tokens, kv heads, pages]
// (paged) or [D, L, kv heads, sequences] (dense), 64 x TT boxes, 128-byte
// swizzle; rows past L read as zeros.  False when a map cannot be made
// (the caller then runs the CUDA-core kernel).
template <typename T>
bool decode_maps(CUtensorMap& mk, CUtensorMap& mv, const DecodeParams& p, bool paged, int D, int TT) {
  const auto fn = tensor_map_encoder();
  if (!fn) return false;
  const int64_t outer = paged ? p.num_pages : p.B;
  const int64_t toks = paged ? p.P : p.L;
  if (outer <= 0 || toks <= 0 || TT > 256) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)toks, (cuuint64_t)p.Hkv, (cuuint64_t)outer};
  const int64_t st[3] = {p.s_tok * 2, p.s_head * 2, p.s0 * 2};
  cuuint64_t strides[3];
  for (int i = 0; i < 3; ++i) {
    if (st[i] <= 0 || (st[i] & 15) || st[i] >= (int64_t(1) << 40)) return false;
    strides[i] = (cuuint64_t)st[i];
  }
  if ((reinterpret_cast<uintptr_t>(p.k) & 15) || (reinterpret_cast<uintptr_t>(p.v) & 15)) return false;
  const cuuint32_t box[4] = {64, (cuuint32_t)TT, 1, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  for (int m = 0; m < 2; ++m) {
    const CUresult r = fn(m == 0 ? &mk : &mv, dt, 4, const_cast<void*>(m == 0 ? p.k : p.v), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  return true;
}

template <typename T, int D, int G, bool PAGED>
int launch_decode(DecodeParams p, const Plan& pl, cudaStream_t st) {
  CUtensorMap mk, mv;
  const bool tc = pl.tc && pl.items > 0 && decode_maps<T>(mk, mv, p, PAGED, D, pl.tile_tokens);
  cudaError_t e = tc ? ensure_smem_limit<decode_mma_kernel<T, D, G, PAGED>>(pl.smem_tc)
                     : ensure_smem_limit<decode_splitkv_kernel<T, D, G, PAGED>>(pl.smem);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  if (PAGED) paged_plan_kernel<<<1, 1024, 0, st>>>(p);
  if (pl.items > 0) {
    ProfileScope prof(st);
    const dim3 grid((unsigned)pl.items), block(kDecodeThreads);
    if (tc) {
      auto kern = decode_mma_kernel<T, D, G, PAGED>;
      if (PAGED)  // after the planner: may start while it runs
        e = launch_dependent(kern, grid, block, pl.smem_tc, st, mk, mv, p);
      else
        kern<<<grid, block, pl.smem_tc, st>>>(mk, mv, p);
    } else {
      auto kern = decode_splitkv_kernel<T, D, G, PAGED>;
      if (PAGED)
        e = launch_dependent(kern, grid, block, pl.smem, st, p);
      else
        kern<<<grid, block, pl.smem, st>>>(p);
    }
    if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(e));
  }
  if (!pl.direct) {  // the merge (also zeros for a dense call over no keys or an empty sequence)
    const unsigned nb = (unsigned)p.B * p.units;
    // long chunk lists (dense: the chunk count; paged: the planner's bound per
    // sequence, on average) are split over 1024 threads, short ones over 256
    const int64_t per_pair = PAGED ? pl.items / std::max(1, p.units) / std::max(1, p.B) : pl.chunks_per_seq;
    const unsigned mthreads = per_pair >= 16 ? 1024u : 256u;
    if (nb > 0) e = launch_dependent(decode_merge_kernel<T, D, G, PAGED>, dim3(nb), dim3(mthreads), 0, st, p);
    if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("decode merge launch: ") + cudaGetErrorString(e));
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(e));
  return AKT_OK;
}

template <typename T, bool PAGED>
int dispatch_decode(DecodeParams p, const Plan& pl, int D, cudaStream_t st) {
#define AKT_G(DD)                                                              \
  switch (pl.G_tile) {                                                         \
    case 1: return launch_decode<T, DD, 1, PAGED>(p, pl, st);                  \
    case 2: return launch_decode<T, DD, 2, PAGED>(p, pl, st);                  \
    case 4: return launch_decode<T, DD, 4, PAGED>(p, pl, st);                  \
    default: break;                                                            \
  }
  switch (D) {
    case 64:
      AKT_G(64)
      if (pl.G_tile == 8) return launch_decode<T, 64, 8, PAGED>(p, pl, st);
      break;
    case 128:
      AKT_G(128)
      if (pl.G_tile == 8) return launch_decode<T, 128, 8, PAGED>(p, pl, st);
      break;
    case 256:
      AKT_G(256)
      break;
  }
#undef AKT_G
  return set_error(AKT_ERR_UNSUPPORTED, "decode: head_dim must be 64, 128 or 256");
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

}  // namespace akt

using namespace akt;

extern "C" {

int akt_abi_version(void) { return AKT_ABI_VERSION; }

const char* akt_last_error(void) { return g_last_error.c_str(); }

int akt_device_status(int device, unsigned int* status_out) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  unsigned int v = 0, vp = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
  if (e == cudaSuccess) e = prefill_status_read(&vp);
  if (v == 0) v = vp;
  cudaSetDevice(prev);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, cudaGetErrorString(e));
  if (status_out) *status_out = v;
  return AKT_OK;
}

int akt_clear_device_status(int device) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  unsigned int z = 0;
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_status, &z, sizeof(z));
  if (e == cudaSuccess) e = prefill_status_clear();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaSetDevice(prev);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, cudaGetErrorString(e));
  return AKT_OK;
}

static int check_common(int B, int Hq, int Hkv, int D, int dtype) {
  if (B < 0 || Hq <= 0 || Hkv <= 0) return set_error(AKT_ERR_INVALID, "batch/heads must be positive");
  if (Hq % Hkv != 0) return set_error(AKT_ERR_INVALID, "num_qo_heads must be a multiple of num_kv_heads");
  if (D != 64 && D != 128 && D != 256) return set_error(AKT_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
  if (dtype != AKT_FLOAT16 && dtype != AKT_BFLOAT16) return set_error(AKT_ERR_INVALID, "dtype");
  return AKT_OK;
}

size_t akt_decode_dense_workspace_size(const akt_decode_dense_args* a) {
  if (!a || check_common(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype) != AKT_OK) return 0;
  Plan pl = make_plan(false, a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->seq_len, 0, 0, 2);
  return pl.ws_bytes;
}

int akt_decode_dense(const akt_decode_dense_args* a, void* ws, size_t ws_bytes, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  int rc = check_common(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype);
  if (rc) return rc;
  if (a->seq_len < 0) return set_error(AKT_ERR_INVALID, "seq_len < 0");
  if (a->q_stride_dim != 1 || a->k_stride_dim != 1 || a->v_stride_dim != 1 || a->k_stride_token != a->head_dim ||
      a->v_stride_token != a->head_dim)
    return set_error(AKT_ERR_UNSUPPORTED, "decode_dense: K/V rows must be contiguous [.., L, D] and q unit-stride");
  if (a->k_stride_batch != a->v_stride_batch || a->k_stride_head != a->v_stride_head)
    return set_error(AKT_ERR_UNSUPPORTED, "decode_dense: K and V must share strides");
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || (a->k_stride_batch % 8) || (a->k_stride_head % 8) ||
      (a->q_stride_batch % 8) || (a->q_stride_head % 8))
    return set_error(AKT_ERR_UNSUPPORTED, "decode_dense: 16-byte alignment required");
  if (a->batch == 0) return AKT_OK;
  Plan pl = make_plan(false, a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->seq_len, 0, 0, 2);
  if (pl.ws_bytes > 0 && (!ws || ws_bytes < pl.ws_bytes)) return set_error(AKT_ERR_WORKSPACE, "decode_dense: workspace too small");
  DecodeParams p{};
  p.q = a->q; p.q_sb = a->q_stride_batch; p.q_sh = a->q_stride_head;
  p.k = a->k; p.v = a->v;
  p.s0 = a->k_stride_batch; p.s_head = a->k_stride_head; p.s_tok = a->k_stride_token;
  p.out = a->out; p.o_sb = a->out_stride_batch; p.o_sh = a->out_stride_head; p.o_sd = a->out_stride_dim;
  p.B = a->batch; p.Hq = a->num_qo_heads; p.Hkv = a->num_kv_heads; p.L = a->seq_len; p.P = 0;
  p.group = p.Hq / p.Hkv; p.g_tiles = p.group / pl.G_tile; p.units = p.Hkv * p.g_tiles;
  p.tile_tokens = pl.tile_tokens; p.chunk_tokens = pl.chunk_tokens; p.chunks_per_seq = pl.chunks_per_seq;
  p.num_stages = pl.num_stages; p.scale_log2 = a->softmax_scale * kLog2e;
  p.direct_out = pl.direct ? 1 : 0;
  if (!pl.direct) {
    p.part_o = reinterpret_cast<float*>(ws);
    p.part_lse = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.off_lse);
  }
  if (a->seq_len == 0) {
    // softmax over no keys: zeros (merge of empty partials)
    p.chunks_per_seq = 0;
    Plan z = pl; z.items = 0; z.direct = false;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->dtype == AKT_FLOAT16) return dispatch_decode<__half, false>(p, z, a->head_dim, st);
    return dispatch_decode<__nv_bfloat16, false>(p, z, a->head_dim, st);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == AKT_FLOAT16) return dispatch_decode<__half, false>(p, pl, a->head_dim, st);
  return dispatch_decode<__nv_bfloat16, false>(p, pl, a->head_dim, st);
}

size_t akt_decode_paged_workspace_size(const akt_decode_paged_args* a) {
  if (!a || check_common(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype) != AKT_OK) return 0;
  if (a->page_size <= 0) return 0;
  Plan pl = make_plan(true, a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, 0, a->page_size,
                      a->num_page_entries, 2);
  return pl.ws_bytes;
}

int akt_decode_paged(const akt_decode_paged_args* a, void* ws, size_t ws_bytes, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  int rc = check_common(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype);
  if (rc) return rc;
  if (a->page_size <= 0) return set_error(AKT_ERR_INVALID, "page_size must be positive");
  if (a->num_page_entries < 0 || a->num_pages < 0) return set_error(AKT_ERR_INVALID, "negative sizes");
  if (a->q_stride_dim != 1 || a->kv_stride_dim != 1 || a->kv_stride_token != a->head_dim)
    return set_error(AKT_ERR_UNSUPPORTED, "decode_paged: page rows must be contiguous [.., P, D] and q unit-stride");
  if (!aligned16(a->q) || !aligned16(a->kv_cache) || (a->kv_stride_page % 8) || (a->kv_stride_kv % 8) ||
      (a->kv_stride_head % 8) || (a->q_stride_batch % 8) || (a->q_stride_head % 8))
    return set_error(AKT_ERR_UNSUPPORTED, "decode_paged: 16-byte alignment required");
  if (a->batch == 0) return AKT_OK;
  Plan pl = make_plan(true, a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, 0, a->page_size,
                      a->num_page_entries, 2);
  if (!ws || ws_bytes < pl.ws_bytes) return set_error(AKT_ERR_WORKSPACE, "decode_paged: workspace too small");
  DecodeParams p{};
  p.q = a->q; p.q_sb = a->q_stride_batch; p.q_sh = a->q_stride_head;
  p.k = a->kv_cache;
  p.v = static_cast<const char*>(a->kv_cache) + a->kv_stride_kv * 2;
  p.s0 = a->kv_stride_page; p.s_head = a->kv_stride_head; p.s_tok = a->kv_stride_token;
  p.indptr = a->kv_page_indptr; p.indices = a->kv_page_indices; p.last_len = a->kv_last_page_len;
  p.num_pages = a->num_pages; p.num_page_entries = a->num_page_entries;
  p.out = a->out; p.o_sb = a->out_stride_batch; p.o_sh = a->out_stride_head; p.o_sd = a->out_stride_dim;
  p.B = a->batch; p.Hq = a->num_qo_heads; p.Hkv = a->num_kv_heads; p.L = 0; p.P = a->page_size;
  p.group = p.Hq / p.Hkv; p.g_tiles = p.group / pl.G_tile; p.units = p.Hkv * p.g_tiles;
  p.tile_tokens = pl.tile_tokens; p.chunk_tokens = pl.chunk_tokens; p.chunks_per_seq = 0;
  p.num_stages = pl.num_stages; p.scale_log2 = a->softmax_scale * kLog2e;
  p.direct_out = 0;
  p.max_chunks = (int)std::min<int64_t>(pl.items / p.units, INT32_MAX - 1);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_lse = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.off_lse);
  p.chunk_offset = reinterpret_cast<int*>(static_cast<char*>(ws) + pl.off_chunk);
  p.tail_seq = p.chunk_offset + (p.B + 2);
  p.tail_rank = p.tail_seq + p.B;
  p.tail_order = p.B <= 1024 ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == AKT_FLOAT16) return dispatch_decode<__half, true>(p, pl, a->head_dim, st);
  return dispatch_decode<__nv_bfloat16, true>(p, pl, a->head_dim, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free paged decode.
//
// Some callers cannot allocate device memory at the point where they run the
// decode: plugin hosts that hand a kernel only its input and output buffers
// (no allocator or workspace hook), and runtimes that plan every byte of
// device memory at start-up and forbid cudaMalloc afterwards (it can
// synchronise the device and fail under a fixed budget).  For them,
// akt_decode_paged_noalloc keeps the split-KV partials in a fixed array that
// the library owns.  The array is a file-scope __device__ variable of
// kNoAllocScratchBytes, so every GPU that loads this library holds that much
// memory until the process exits.  Its host-side name is only a stand-in for
// the device symbol: host code must use the address cudaGetSymbolAddress
// returns for the current device, never the name itself.
// ---------------------------------------------------------------------------
namespace akt {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};

// The driver's current context, through the runtime's entry-point query (the
// library links only the runtime).  Null if the query is unavailable.
CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
               ? reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f)
               : nullptr;
  }();
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

// Device address of the scratch array on the current device.  It is looked up
// on the first call on a device, and again whenever the context current at the
// call differs from the one it was looked up under (a caller on its own
// driver-API context gets that context's copy of the module).  A device reset
// (cudaDeviceReset) unloads the module; the address cached before it is not
// detected as stale, so a process that resets a device must not call this
// entry point on that device afterwards.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(AKT_ERR_INVALID, "device ordinal out of range");
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return set_error(AKT_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
    g_noalloc_ctx[dev] = current_context();  // the runtime call above may have made the primary context current
  }
  *out = g_noalloc_ptr[dev];
  return AKT_OK;
}

}  // namespace
}  // namespace akt

extern "C" int akt_decode_paged_noalloc(const akt_decode_paged_args* a, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  int rc = check_common(a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, a->dtype);
  if (rc) return rc;
  if (a->page_size <= 0) return set_error(AKT_ERR_INVALID, "page_size must be positive");
  if (a->num_page_entries < 0 || a->num_pages < 0) return set_error(AKT_ERR_INVALID, "negative sizes");
  if (a->q_stride_dim != 1 || a->kv_stride_dim != 1 || a->kv_stride_token != a->head_dim)
    return set_error(AKT_ERR_UNSUPPORTED, "decode_paged_noalloc: page rows must be contiguous [.., P, D] and q unit-stride");
  if (!aligned16(a->q) || !aligned16(a->kv_cache) || (a->kv_stride_page % 8) || (a->kv_stride_kv % 8) ||
      (a->kv_stride_head % 8) || (a->q_stride_batch % 8) || (a->q_stride_head % 8))
    return set_error(AKT_ERR_UNSUPPORTED, "decode_paged_noalloc: 16-byte alignment required");
  if (a->batch == 0) return AKT_OK;
  Plan pl = make_plan(true, a->batch, a->num_qo_heads, a->num_kv_heads, a->head_dim, 0, a->page_size,
                      a->num_page_entries, 2);
  // Same kernels as akt_decode_paged.  When the partials of the default split
  // do not fit the fixed array, use longer chunks (fewer partials) until they do.
  const int units = a->num_kv_heads * (a->num_qo_heads / a->num_kv_heads / pl.G_tile);
  while (pl.ws_bytes > kNoAllocScratchBytes && pl.chunk_tokens < (1 << 20)) {
    pl.chunk_tokens *= 2;
    layout_workspace(pl, true, a->batch, units, a->head_dim, 0, a->page_size, a->num_page_entries);
  }
  if (pl.ws_bytes > kNoAllocScratchBytes)
    return set_error(AKT_ERR_WORKSPACE, "decode_paged_noalloc: this call needs " + std::to_string(pl.ws_bytes) +
                                            " bytes of scratch; the allocation-free entry point holds at most " +
                                            std::to_string(kNoAllocScratchBytes) + " bytes");
  void* ws = nullptr;
  rc = noalloc_scratch(&ws);
  if (rc) return rc;
  DecodeParams p{};
  p.q = a->q; p.q_sb = a->q_stride_batch; p.q_sh = a->q_stride_head;
  p.k = a->kv_cache;
  p.v = static_cast<const char*>(a->kv_cache) + a->kv_stride_kv * 2;
  p.s0 = a->kv_stride_page; p.s_head = a->kv_stride_head; p.s_tok = a->kv_stride_token;
  p.indptr = a->kv_page_indptr; p.indices = a->kv_page_indices; p.last_len = a->kv_last_page_len;
  p.num_pages = a->num_pages; p.num_page_entries = a->num_page_entries;
  p.out = a->out; p.o_sb = a->out_stride_batch; p.o_sh = a->out_stride_head; p.o_sd = a->out_stride_dim;
  p.B = a->batch; p.Hq = a->num_qo_heads; p.Hkv = a->num_kv_heads; p.L = 0; p.P = a->page_size;
  p.group = p.Hq / p.Hkv; p.g_tiles = p.group / pl.G_tile; p.units = p.Hkv * p.g_tiles;
  p.tile_tokens = pl.tile_tokens; p.chunk_tokens = pl.chunk_tokens; p.chunks_per_seq = 0;
  p.num_stages = pl.num_stages; p.scale_log2 = a->softmax_scale * kLog2e;
  p.direct_out = 0;
  p.max_chunks = (int)std::min<int64_t>(pl.items / p.units, INT32_MAX - 1);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_lse = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.off_lse);
  p.chunk_offset = reinterpret_cast<int*>(static_cast<char*>(ws) + pl.off_chunk);
  p.tail_seq = p.chunk_offset + (p.B + 2);
  p.tail_rank = p.tail_seq + p.B;
  p.tail_order = p.B <= 1024 ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == AKT_FLOAT16) return dispatch_decode<__half, true>(p, pl, a->head_dim, st);
  return dispatch_decode<__nv_bfloat16, true>(p, pl, a->head_dim, st);
}
