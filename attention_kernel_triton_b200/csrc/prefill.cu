// Causal / non-causal GQA prefill (flash-attention forward) for sm_100a on the
// 5th-generation tensor cores (tcgen05 + TMEM), with padded var-len support.
//
// Replaces the Triton kernels of prefill_flash_attention.py:109-335 and
// prefill_flash_attention_var_len_padding.py:109-341.  Same math:
// O = softmax(Q K^T * s [+ top-left causal mask]) V with GQA kv head h / G,
// fp32 accumulation, P rounded to the input dtype before P.V (PF:94); the
// var-len variant skips query rows past each sequence's length (PV:186-187)
// and masks no keys beyond the causal mask (the reference does not either).
//
// Persistent CTAs (one per SM) walk a list of work items, heaviest causal
// tiles first.  An item is two 128-row query tiles ("slots") that read the
// same K/V: two qo heads of one kv head at the same rows when the GQA group
// is even, else two consecutive query tiles of one head.  Warp roles:
//   warps 0-3 / 4-7  softmax warpgroup of slot 0 / 1: thread i owns query row
//              i = TMEM lane i; reads S with tcgen05.ld, writes P (input
//              dtype) back to TMEM with tcgen05.st, rescales O in TMEM when
//              its running max moves, and writes the normalised output.
//   warp 8     TMA producer of Q and the K ring; warp 10 of the V ring.
//   warp 9     TMEM allocator; its lane 0 issues slot 0's MMAs, lane 0 of
//              warp 11 those of slot 1:
//              S_t = Q_t K_j^T (M=128, N=BN, K=D; A and B in shared memory)
//              O_t += P_t V_j   (M=128, N=D,  K=BN; A = P in TMEM, B = V)
// TMEM (512 columns): S[2] (BN each), O[2] (D each), P[2] (BN/2 each, two
// 16-bit values per column).  With S and P apart, S for key tile j+1 is
// computed while the softmax still works on tile j; the only per-tile wait
// of a softmax warpgroup is for its previous P.V before it overwrites P.
// The third warpgroup's spare registers go to the softmax warpgroups
// (setmaxnreg).
//
// The running max used for exponentiation only moves when the row max grows
// by more than 8 (log2 units), so O is rescaled rarely (P <= 2^8 stays exact
// enough in fp16/bf16 relative terms; the final O/l is unchanged).  At
// head_dim 64 MUFU ex2 (16 results per clock per SM, 256 flops of the two
// MMAs per result) is the busiest pipe, but the kernel is bound by its
// per-tile chain: S MMA -> softmax -> P -> P.V MMA -> next P, with about 100
// cycles of issue per MMA and about 460 cycles from a commit to the waiting
// thread; removing every exponential speeds it up by only 11 %.
// Built without -rdc (whole-program device code): with relocatable device
// code ptxas ignores setmaxnreg, and the softmax warpgroups need its budget.
#define AKT_WHOLE_PROGRAM 1
#include "common.cuh"
#include "profile.cuh"
#include "tensor_map.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdlib>
#include <mutex>
#include <string>

namespace akt {

int set_error(int code, const std::string& msg);

namespace {

constexpr int BM = 128;            // query rows per slot
constexpr int kSlots = 2;          // query tiles per work item
constexpr int kThreads = 384;      // 2 softmax warpgroups + a warpgroup holding the producer and MMA warps
constexpr int kLoadWarp = 8;       // Q and the K ring
constexpr int kMmaWarp = 9;
constexpr int kLoadVWarp = 10;     // the V ring (its own warp: two waiting lanes of one warp stall each other)
constexpr int kMmaWarp1 = 11;      // MMA issuer of slot 1 (slot 0: kMmaWarp)
// Register split: the kernel is compiled for 168 registers per thread (3 warps
// per SM sub-partition); the producer/MMA warpgroup gives registers back and
// the softmax warpgroups take them: 2*128*216 + 128*64 <= 384*168 (224 and 56
// for the variant that also writes the log-sum-exp).
constexpr int kLaunchRegs = 168;
template <bool LSE>
struct RegSplit {
  static constexpr int softmax = LSE ? 224 : 216;
  static constexpr int control = LSE ? 56 : 64;
  static_assert(2 * 128 * softmax + 128 * control <= kThreads * kLaunchRegs, "register split");
};
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Var-len work order (shared memory, built by every CTA in its prologue from
// the per-sequence lengths).  With padding, a query tile past its sequence's
// length costs nothing, and the plain order (query-tile index, then batch)
// scatters those free items among the real ones, so the per-CTA sums of item
// costs come out uneven.  Here the list is grouped into levels, one per
// query-tile index (paired heads) or pair of query tiles (one head per item),
// from the last down; the causal cost of a real item grows with its level.
// Level l holds the real items of the batches that reach it, the longest
// sequences first (perm); every free item follows all real ones, in the same
// level order.
// The order is a compile-time variant (SCHED), used only by var-len calls that
// fit the table: the other kernels compile exactly as without it (extra item
// setup code in the softmax warps' region, at 216 registers, measured 9 %
// slower on the causal prefill even where it never ran).  The table is kept
// small (2.3 KB), so D=64 stays inside the 164 KB shared-memory carveout.
constexpr int kSchedMaxB = 256;      // batches the table holds
constexpr int kSchedMaxTiles = 128;  // levels the table holds (S <= 16384, or 32768 with one head per item)
struct VarlenSched {
  int32_t vstart[kSchedMaxTiles + 1];  // first real item of level l
  int32_t zstart[kSchedMaxTiles + 1];  // first free item of level l, counted after the last real item
  int16_t cnt[kSchedMaxTiles];         // batches with a real item at level l
  int16_t perm[kSchedMaxB];            // batches by levels reached, descending (ties by index)
  int16_t ntiles[kSchedMaxB];          // levels each sequence reaches (its query tiles, or tile pairs)
};

// Tile configuration per head_dim D.  Keys per tile BN is chosen so that
// S[2], O[2] and P[2] fit the 512 TMEM columns of one SM:
//   D=64 : BN=128 -> 256 + 128 + 128 = 512 columns; smem 64 KB Q + 3-stage K, V rings = 160 KB
//   D=128: BN=64  -> 128 + 256 +  64 = 448 columns; smem 128 KB Q + 2-stage rings = 192 KB
template <int D>
struct Cfg {
  static constexpr int BN = D == 64 ? 128 : 64;
  static constexpr int DB = D / 64;                       // 64-element (128 B) swizzle blocks per row
  static constexpr int COL_S = 0;                         // + slot * BN
  static constexpr int COL_O = 2 * BN;                    // + slot * D
  static constexpr int COL_P = 2 * BN + 2 * D;            // + slot * BN / 2
  static constexpr int TMEM_COLS = 512;
  static_assert(COL_P + BN <= TMEM_COLS, "TMEM budget");
  static constexpr int NQ = 2;                            // Q buffers per slot (next item's Q loads early)
  static constexpr int NSK = D == 64 ? 3 : 2, NSV = NSK;  // K / V ring stages
  static constexpr uint32_t Q_BYTES = BM * D * 2;         // one slot
  static constexpr uint32_t KV_BYTES = BN * D * 2;        // one K or V tile
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + kSlots * NQ * Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + NSK * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + NSV * KV_BYTES;
  // mbarriers: q_full/q_empty [slot][NQ], k and v full/empty rings, s_full,
  // s_empty, p_full, pv_done [slot], mma_idle; then the TMEM address word and
  // the abort flag
  static constexpr int N_BARS = 2 * kSlots * NQ + 2 * NSK + 2 * NSV + 4 * kSlots + 1;
  static constexpr uint32_t BAR_BYTES = (N_BARS * 8 + 8 + 15) / 16 * 16;
  static constexpr uint32_t SMEM = OFF_BAR + BAR_BYTES;  // base is 1024-aligned
  // the var-len order table follows, in the kernels that use it
  static constexpr uint32_t OFF_SCHED = SMEM;
  static constexpr uint32_t SMEM_SCHED = SMEM + sizeof(VarlenSched);
  static_assert(SMEM_SCHED <= 227 * 1024, "shared memory budget");
  // with the 1 KB the driver reserves per CTA, D=64 fits the 164 KB carveout
  static_assert(D != 64 || SMEM_SCHED + 1024 <= 164 * 1024, "D=64 shared-memory carveout");
};

struct PrefillParams {
  void* o;
  int64_t o_sb, o_sh, o_ss;  // element strides (dim stride 1)
  const int32_t* varlen;     // [B] or null
  int B, Hq, Hkv, S, group;
  int n_q_tiles;
  int n_items;
  int pair_heads;            // 1: slots are qo heads 2p, 2p+1 at the same rows; 0: query tiles 2p, 2p+1 of one head
  int causal;
  float scale_log2;
  float* lse;                // [B, Hq, S] natural-log sum-exp per row, or null
  int64_t lse_sb, lse_sh;
};

// One work item: the key-tile count of each slot (0 = slot has no valid rows).
struct Item {
  int b, kvh, seq_len, L;
  int h[kSlots], q0[kSlots], nkv[kSlots];
};

// The CTA's k-th item: rounds of gridDim.x items in list order, taken left to
// right in even rounds and right to left in odd ones, so the per-CTA sums of
// the (descending) item costs stay even; -1 past the end of the list.
__device__ __forceinline__ int item_of(const PrefillParams& p, int k) {
  const int g = gridDim.x;
  const int i = k * g + ((k & 1) ? g - 1 - (int)blockIdx.x : (int)blockIdx.x);
  return i < p.n_items ? i : -1;
}

// Item i of the list; every role of the CTA decodes the same item.  Items are
// ordered by query-tile index, last (longest causal row range) first.
// Level of item i in a table of level starts (st[0] = 0 <= i < st[n]): the l
// with st[l] <= i < st[l + 1].  A linear scan (few live registers: the
// producer and MMA warps decode every item with 56-64 registers); at most
// n_q_tiles steps, against an item of up to n_q_tiles key tiles.
__device__ __forceinline__ int sched_level(const int32_t* st, int i) {
  int l = 0;
  while (st[l + 1] <= i) ++l;
  return l;
}

// Fills the var-len order table (all threads of the CTA; the caller's next
// __syncthreads publishes the prefix sums thread 0 writes last).
// Levels of the order: query tiles (paired heads) or pairs of consecutive
// query tiles (one head per item); the items of a (level, batch) class: head
// pairs or heads.
__device__ __forceinline__ int sched_levels(const PrefillParams& p) {
  return p.pair_heads ? p.n_q_tiles : (p.n_q_tiles + 1) / 2;
}
__device__ __forceinline__ int sched_class_items(const PrefillParams& p) { return p.pair_heads ? p.Hq / 2 : p.Hq; }

__device__ __forceinline__ void build_sched(const PrefillParams& p, VarlenSched* vs) {
  for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
    const int len = min(max(__ldg(p.varlen + b), 0), p.S);
    const int nt = (len + BM - 1) / BM;
    vs->ntiles[b] = (int16_t)(p.pair_heads ? nt : (nt + 1) / 2);  // levels the sequence reaches
  }
  __syncthreads();
  for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
    const int nb = vs->ntiles[b];
    int rank = 0;
    for (int o = 0; o < p.B; ++o) {
      const int no = vs->ntiles[o];
      rank += (no > nb || (no == nb && o < b)) ? 1 : 0;
    }
    vs->perm[rank] = (int16_t)b;
  }
  const int n_lev = sched_levels(p);
  for (int l = threadIdx.x; l < n_lev; l += blockDim.x) {
    const int lev = n_lev - 1 - l;
    int c = 0;
    for (int o = 0; o < p.B; ++o) c += vs->ntiles[o] > lev ? 1 : 0;
    vs->cnt[l] = (int16_t)c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int per_cls = sched_class_items(p);
    int v = 0, z = 0;
    for (int l = 0; l < n_lev; ++l) {
      vs->vstart[l] = v;
      vs->zstart[l] = z;
      v += vs->cnt[l] * per_cls;
      z += (p.B - vs->cnt[l]) * per_cls;
    }
    vs->vstart[n_lev] = v;
    vs->zstart[n_lev] = z;
  }
}

// Item i of the var-len order: level index l (counted from the last level),
// batch and index inside its class.
__device__ __forceinline__ void sched_item(const PrefillParams& p, const VarlenSched* vs, int i, int& l, int& b,
                                           int& k) {
  const int per_cls = sched_class_items(p);
  const int vtot = vs->vstart[sched_levels(p)];
  int r, first;
  if (i < vtot) {
    l = sched_level(vs->vstart, i);
    r = i - vs->vstart[l];
    first = 0;
  } else {
    l = sched_level(vs->zstart, i - vtot);
    r = i - vtot - vs->zstart[l];
    first = vs->cnt[l];
  }
  b = vs->perm[first + r / per_cls];
  k = r % per_cls;
}

template <bool SCHED>
__device__ __forceinline__ Item decode_item(const PrefillParams& p, const VarlenSched* vs, int i, int BN) {
  Item it;
  if (p.pair_heads) {
    const int hp_n = p.Hq / 2;
    int qt, hp;
    if constexpr (SCHED) {
      int l;
      sched_item(p, vs, i, l, it.b, hp);
      qt = p.n_q_tiles - 1 - l;
    } else {
      const int per = p.B * hp_n;
      qt = p.n_q_tiles - 1 - i / per;
      const int r = i % per;
      it.b = r / hp_n;
      hp = r % hp_n;
    }
    it.h[0] = 2 * hp;
    it.h[1] = 2 * hp + 1;
    it.q0[0] = it.q0[1] = qt * BM;
  } else if constexpr (SCHED) {
    int l, h;
    sched_item(p, vs, i, l, it.b, h);
    const int qp = (p.n_q_tiles + 1) / 2 - 1 - l;
    it.h[0] = it.h[1] = h;
    it.q0[0] = 2 * qp * BM;
    it.q0[1] = (2 * qp + 1) * BM;
  } else {
    const int per = p.B * p.Hq, n_qp = (p.n_q_tiles + 1) / 2;
    const int qp = n_qp - 1 - i / per, r = i % per;
    it.b = r / p.Hq;
    it.h[0] = it.h[1] = r % p.Hq;
    it.q0[0] = 2 * qp * BM;
    it.q0[1] = (2 * qp + 1) * BM;
  }
  it.kvh = it.h[0] / p.group;
  it.seq_len = p.varlen ? min(max(__ldg(p.varlen + it.b), 0), p.S) : p.S;
  it.L = 0;
#pragma unroll
  for (int t = 0; t < kSlots; ++t) {
    // causal: rows past seq_len are zeroed, so keys past it are never needed
    const int last_key = p.causal ? min(it.q0[t] + BM, it.seq_len) - 1 : p.S - 1;
    it.nkv[t] = it.q0[t] < it.seq_len ? last_key / BN + 1 : 0;
    it.L = max(it.L, it.nkv[t]);
  }
  return it;
}

// -------------------------------------------------------------------------
// PTX helpers
// -------------------------------------------------------------------------
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

__host__ __device__ constexpr uint32_t idesc_f16(int fmt, int M, int N, int b_mn_major) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// A shared-memory descriptor as its two 32-bit words.  The low word holds the
// start address in 16-byte units (bits 0-13) and the leading byte offset; the
// high word the stride byte offset, version and swizzle.  Shared addresses
// stay below 2^18 bytes, so a tile offset is one add on the low word, which
// keeps the issuing thread's work per MMA small.
struct Desc {
  uint32_t lo, hi;
};

__device__ __forceinline__ Desc desc_words(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  const uint64_t d = desc_sw128(saddr, lbo, sbo);
  return Desc{(uint32_t)d, (uint32_t)(d >> 32)};
}

// A and B from shared memory (descriptor words a_lo/a_hi, b_lo/b_hi)
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                        uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(tmem_d),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
      : "memory");
}

// A operand from TMEM (K-major, two 16-bit values per 32-bit column, row i
// in lane i), B from shared memory through its descriptor words
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint32_t b_lo, uint32_t b_hi,
                                           uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <typename T>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
  return Elem<T>::pack2(a, b);
}

// O row of one softmax thread (D fp32 TMEM columns at tO) into registers:
// all loads issued, then one wait.
template <int D>
__device__ __forceinline__ void read_o(uint32_t tO, uint32_t (&o)[D / 32][32]) {
#pragma unroll
  for (int c = 0; c < D / 32; ++c) tmem_ld32(tO + c * 32, o[c]);
  tmem_wait_ld();
}

// Normalised output row: o times inv, converted to T, packed two per word.
template <typename T, int D>
__device__ __forceinline__ void pack_o(const uint32_t (&o)[D / 32][32], float inv, uint32_t (&w)[D / 2]) {
#pragma unroll
  for (int c = 0; c < D / 32; ++c)
#pragma unroll
    for (int e = 0; e < 32; e += 2)
      w[(c * 32 + e) / 2] = Elem<T>::pack2(__uint_as_float(o[c][e]) * inv, __uint_as_float(o[c][e + 1]) * inv);
}

// Packed output row to orow (null: rows past S, not stored), 16 bytes a store.
template <typename T, int D>
__device__ __forceinline__ void store_o(const uint32_t (&w)[D / 2], T* orow) {
  if (!orow) return;
#pragma unroll
  for (int c = 0; c < D / 8; ++c)
    reinterpret_cast<uint4*>(orow)[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Slow path of a bounded mbarrier wait: spins on try_wait; every 256 polls it
// gives up if another role of the CTA has aborted, or, after kWaitLimitNs,
// records kStatusWaitTimeout and raises the abort flag itself.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(kStatusWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// -------------------------------------------------------------------------
// kernel
// -------------------------------------------------------------------------
template <typename T, int D, bool LSE, bool SCHED>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const PrefillParams p) {
  using C = Cfg<D>;
  constexpr int BN = C::BN;
  constexpr int fmt = std::is_same<T, __half>::value ? 0 : 1;
  constexpr uint32_t IDESC_S = idesc_f16(fmt, BM, BN, 0);
  constexpr uint32_t IDESC_PV = idesc_f16(fmt, BM, D, 1);

  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023u) {  // swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_status(kStatusWaitTimeout);
    return;
  }
  if constexpr (SCHED) build_sched(p, reinterpret_cast<VarlenSched*>(smem + C::OFF_SCHED));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;                       // [slot][NQ]
  uint64_t* q_empty = q_full + kSlots * C::NQ;   // [slot][NQ]
  uint64_t* k_full = q_empty + kSlots * C::NQ;   // [NSK]
  uint64_t* k_empty = k_full + C::NSK;           // [NSK]
  uint64_t* v_full = k_empty + C::NSK;           // [NSV]
  uint64_t* v_empty = v_full + C::NSV;           // [NSV]
  uint64_t* s_full = v_empty + C::NSV;           // [slot]
  uint64_t* s_empty = s_full + kSlots;           // [slot]
  uint64_t* p_full = s_empty + kSlots;           // [slot]
  uint64_t* pv_done = p_full + kSlots;           // [slot]
  uint64_t* mma_idle = pv_done + kSlots;         // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_idle + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int t = 0; t < kSlots; ++t) {
      for (int q = 0; q < C::NQ; ++q) {
        mbar_init(&q_full[t * C::NQ + q], 1);
        mbar_init(&q_empty[t * C::NQ + q], 1);
      }
      mbar_init(&s_full[t], 1);
      mbar_init(&s_empty[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&pv_done[t], 1);
    }
    for (int s = 0; s < C::NSK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], kSlots);  // one commit per slot's MMA issuer
    }
    for (int s = 0; s < C::NSV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], kSlots);
    }
    mbar_init(mma_idle, kSlots);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // A completed phase costs one try_wait (~20 cycles); the abort flag and the
  // time limit are only looked at while spinning, because a shared-memory
  // load ahead of every try_wait costs ~10x that on the issuing thread.
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    return wait_or_abort(bar, parity, abort_flag);
  };

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<LSE>::control));
  if (warp == kLoadWarp || warp == kLoadVWarp) {
    // ========================= TMA producers =========================
    // Phases continue across items: counters are global to the CTA.  Q load n
    // of a slot goes to buffer n % NQ.
    if (warp == kLoadWarp && lane == 0) {
      uint32_t qn[kSlots] = {0, 0}, gk = 0;
      bool ok = true;
      for (int k = 0, i = item_of(p, 0); ok && i >= 0; i = item_of(p, ++k)) {
        const Item it = decode_item<SCHED>(p, reinterpret_cast<const VarlenSched*>(smem + C::OFF_SCHED), i, BN);
#pragma unroll
        for (int t = 0; t < kSlots; ++t) {
          if (!it.nkv[t]) continue;
          const uint32_t qb = qn[t] % C::NQ, use = qn[t] / C::NQ;
          // buffer qb is free once the last S MMA that read it (NQ loads ago) is done
          if (use && !wait(&q_empty[t * C::NQ + qb], (use - 1) & 1)) { ok = false; break; }
          unsigned char* sQ = smem + C::OFF_Q + (t * C::NQ + qb) * C::Q_BYTES;
          mbar_arrive_expect_tx(&q_full[t * C::NQ + qb], C::Q_BYTES);
#pragma unroll
          for (int db = 0; db < C::DB; ++db)
            tma_load_4d(sQ + db * BM * 128, &tmQ, db * 64, it.q0[t], it.h[t], it.b, &q_full[t * C::NQ + qb]);
          ++qn[t];
        }
        for (int j = 0; ok && j < it.L; ++j, ++gk) {
          const uint32_t st = gk % C::NSK;
          if (gk >= C::NSK && !wait(&k_empty[st], ((gk / C::NSK) - 1) & 1)) { ok = false; break; }
          unsigned char* sK = smem + C::OFF_K + st * C::KV_BYTES;
          mbar_arrive_expect_tx(&k_full[st], C::KV_BYTES);
#pragma unroll
          for (int db = 0; db < C::DB; ++db)
            tma_load_4d(sK + db * BN * 128, &tmK, db * 64, j * BN, it.kvh, it.b, &k_full[st]);
        }
      }
      if (*abort_flag) {  // drain loads still in flight into this CTA's shared memory
        for (int t = 0; t < kSlots; ++t)
          for (uint32_t n = qn[t] > C::NQ ? qn[t] - C::NQ : 0; n < qn[t]; ++n)
            mbar_wait(&q_full[t * C::NQ + n % C::NQ], (n / C::NQ) & 1);
        for (uint32_t g = gk > C::NSK ? gk - C::NSK : 0; g < gk; ++g) mbar_wait(&k_full[g % C::NSK], (g / C::NSK) & 1);
      }
    } else if (warp == kLoadVWarp && lane == 0) {
      uint32_t gv = 0;
      bool ok = true;
      for (int k = 0, i = item_of(p, 0); ok && i >= 0; i = item_of(p, ++k)) {
        const Item it = decode_item<SCHED>(p, reinterpret_cast<const VarlenSched*>(smem + C::OFF_SCHED), i, BN);
        for (int j = 0; j < it.L; ++j, ++gv) {
          const uint32_t st = gv % C::NSV;
          if (gv >= C::NSV && !wait(&v_empty[st], ((gv / C::NSV) - 1) & 1)) { ok = false; break; }
          unsigned char* sV = smem + C::OFF_V + st * C::KV_BYTES;
          mbar_arrive_expect_tx(&v_full[st], C::KV_BYTES);
#pragma unroll
          for (int db = 0; db < C::DB; ++db)
            tma_load_4d(sV + db * BN * 128, &tmV, db * 64, j * BN, it.kvh, it.b, &v_full[st]);
        }
      }
      if (*abort_flag) {
        for (uint32_t g = gv > C::NSV ? gv - C::NSV : 0; g < gv; ++g) mbar_wait(&v_full[g % C::NSV], (g / C::NSV) & 1);
      }
    }
  } else if ((warp == kMmaWarp || warp == kMmaWarp1) && lane == 0) {
    // ========================= MMA issuers =========================
    // One thread per slot issues that slot's MMAs and commits, so neither
    // slot's next S waits behind the other slot's P.V.  Each issuer walks all
    // key tiles of every item: it waits for each K and V stage and commits
    // one arrival to its release barrier (count 2) even for tiles its slot
    // skips.  Per tile: S of tile j, then P.V of tile j-1, so the next S is
    // queued before the tensor core waits on the softmax, also across items.
    const int t = warp == kMmaWarp ? 0 : 1;
    // descriptors of the first Q buffer of this slot and of the first K and V
    // stages; buffers and k-steps are offsets on the low word
    const Desc dq = desc_words(smem_u32(smem + C::OFF_Q + t * C::NQ * C::Q_BYTES), 16, 1024);
    const Desc dk = desc_words(smem_u32(smem + C::OFF_K), 16, 1024);
    const Desc dv = desc_words(smem_u32(smem + C::OFF_V), BN * 128, 1024);
    // ring positions as (stage, phase bit), advanced without divisions
    uint32_t kst = 0, kph = 0, vst = 0, vph = 0, qn = 0, sc = 0, pc = 0;
    bool ok = true;
    bool pend = false, pend_act = false, pend_first = false;  // P.V owed for the previous tile
    auto issue_pv = [&]() -> bool {
      const uint32_t st = vst;
      if (!wait(&v_full[st], vph)) return false;
      if (pend_act) {
        if (!wait(&p_full[t], pc & 1)) return false;
        tc_fence_after();
        const uint32_t v_lo = dv.lo + st * (C::KV_BYTES >> 4);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          mma_f16_ts(tmem + C::COL_O + t * D, tmem + C::COL_P + t * (BN / 2) + k * 8, v_lo + k * (2048 >> 4), dv.hi,
                     IDESC_PV, (!pend_first || k > 0) ? 1u : 0u);
        mma_commit(&pv_done[t]);
        ++pc;
      }
      mma_commit(&v_empty[st]);
      if (++vst == C::NSV) { vst = 0; vph ^= 1u; }
      return true;
    };
    for (int k = 0, i = item_of(p, 0); ok && i >= 0; i = item_of(p, ++k)) {
      const Item it = decode_item<SCHED>(p, reinterpret_cast<const VarlenSched*>(smem + C::OFF_SCHED), i, BN);
      const int nkv = t ? it.nkv[1] : it.nkv[0];
      for (int j = 0; ok && j < it.L; ++j) {
        const uint32_t st = kst;
        if (!wait(&k_full[st], kph)) { ok = false; break; }
        if (j < nkv) {
          const uint32_t qb = qn % C::NQ, use = qn / C::NQ;
          if (j == 0 && !wait(&q_full[t * C::NQ + qb], use & 1)) { ok = false; break; }
          if (sc && !wait(&s_empty[t], (sc - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t q_lo = dq.lo + qb * (C::Q_BYTES >> 4), k_lo = dk.lo + st * (C::KV_BYTES >> 4);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t offq = (k >> 2) * (BM * 128) + (k & 3) * 32;
            const uint32_t offk = (k >> 2) * (BN * 128) + (k & 3) * 32;
            mma_f16(tmem + C::COL_S + t * BN, q_lo + (offq >> 4), dq.hi, k_lo + (offk >> 4), dk.hi, IDESC_S, k > 0);
          }
          mma_commit(&s_full[t]);
          if (j == nkv - 1) {
            mma_commit(&q_empty[t * C::NQ + qb]);
            ++qn;
          }
          ++sc;
        }
        mma_commit(&k_empty[st]);
        if (++kst == C::NSK) { kst = 0; kph ^= 1u; }
        if (pend && !issue_pv()) { ok = false; break; }
        pend = true;
        pend_first = j == 0;
        pend_act = j < nkv;
      }
    }
    if (ok && pend) issue_pv();
    // every MMA issued by this thread has finished before the CTA can exit
    mma_commit(mma_idle);
    mbar_wait(mma_idle, 0);
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(RegSplit<LSE>::softmax));
    // ========================= softmax warpgroups =========================
    const int t = warp >> 2;                   // slot
    const int r = threadIdx.x & (BM - 1);      // row in the tile = TMEM lane
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_addr + C::COL_S + t * BN;
    const uint32_t tO = tmem + lane_addr + C::COL_O + t * D;
    const uint32_t tP = tmem + lane_addr + C::COL_P + t * (BN / 2);
    uint32_t sc = 0, pc = 0, pn = 0;           // S tiles read, P.V completions seen, P tiles written
    // The output of an item is read from TMEM after the first tile of the next
    // one has been exponentiated (so the wait for the item's last P.V is
    // hidden) and stored to global memory after that tile's P is handed to
    // the MMA issuer (so the stores are off the P -> P.V path).
    T* pend_orow = nullptr;
    float pend_inv = 0.f;
    bool ok = true, pend_out = false;
    for (int k = 0, i = item_of(p, 0); ok && i >= 0; i = item_of(p, ++k)) {
      const Item it = decode_item<SCHED>(p, reinterpret_cast<const VarlenSched*>(smem + C::OFF_SCHED), i, BN);
      // slot fields selected without dynamic indexing (keeps Item in registers)
      const int q0 = t ? it.q0[1] : it.q0[0], hq = t ? it.h[1] : it.h[0], nkv = t ? it.nkv[1] : it.nkv[0];
      const int row = q0 + r;
      T* orow = static_cast<T*>(p.o) + (int64_t)it.b * p.o_sb + (int64_t)hq * p.o_sh + (int64_t)row * p.o_ss;
      if (!nkv) {  // slot entirely past the sequence (var-len padding): zeros
        if (row < p.S) {
#pragma unroll
          for (int c = 0; c < D; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
          if constexpr (LSE) p.lse[(int64_t)it.b * p.lse_sb + (int64_t)hq * p.lse_sh + row] = -INFINITY;
        }
        continue;
      }
      float m_use = -INFINITY, l = 0.f;
      for (int j = 0; j < nkv; ++j) {
        if (!wait(&s_full[t], sc & 1)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        float x[BN];
        {
          uint32_t rr[BN / 32][32];
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, rr[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(rr[c][e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[t]);
        // masks only where a key tile reaches past the tile's first row (causal
        // diagonal) or past S
        const bool masked = (p.causal && (j + 1) * BN - 1 > q0) || (j + 1) * BN > p.S;
        if (masked) {
          const int lim = min(p.causal ? row : p.S - 1, p.S - 1) - j * BN;  // last visible column
#pragma unroll
          for (int c = 0; c < BN; ++c) x[c] = c > lim ? -INFINITY : x[c];
        }
        // row max of the raw scores (scale > 0): 4 chains of 3-input max
        float mx;
        {
          float a0 = fmaxf(x[0], x[4]), a1 = fmaxf(x[1], x[5]), a2 = fmaxf(x[2], x[6]), a3 = fmaxf(x[3], x[7]);
#pragma unroll
          for (int c = 8; c < BN; c += 8) {
            a0 = max3f(a0, x[c + 0], x[c + 1]);
            a1 = max3f(a1, x[c + 2], x[c + 3]);
            a2 = max3f(a2, x[c + 4], x[c + 5]);
            a3 = max3f(a3, x[c + 6], x[c + 7]);
          }
          mx = max3f(a0, a1, fmaxf(a2, a3)) * p.scale_log2;
        }
        const float m_new = fmaxf(m_use, mx);
        const bool need = m_new > m_use + kRescaleThreshold || (m_use == -INFINITY && m_new != -INFINITY);
        float alpha = 1.f;
        if (need) {
          alpha = fast_exp2(m_use - m_new);
          m_use = m_new;
        }
        const float m_sub = m_use == -INFINITY ? 0.f : m_use;
        // P = 2^(s*scale - m), packed to the input dtype
        const float2 sl2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_sub, -m_sub);
        float2 rs2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) rs2[e] = make_float2(0.f, 0.f);
        uint32_t pk[BN / 64][32];
#pragma unroll
        for (int e = 0; e < BN / 2; ++e) {
          const float2 v = ffma2(make_float2(x[2 * e], x[2 * e + 1]), sl2, nm2);
          const float2 ev = make_float2(fast_exp2(v.x), fast_exp2(v.y));
          rs2[e & 3] = __fadd2_rn(rs2[e & 3], ev);
          pk[e >> 5][e & 31] = pack_p<T>(ev.x, ev.y);
        }
        const float2 rs01 = __fadd2_rn(rs2[0], rs2[1]), rs23 = __fadd2_rn(rs2[2], rs2[3]);
        const float2 rsum = __fadd2_rn(rs01, rs23);
        l = l * alpha + (rsum.x + rsum.y);
        // P_t and O_t are free once the previous P.V of this slot is done
        if (pn) {
          if (!wait(&pv_done[t], pc & 1)) { ok = false; break; }
          ++pc;
          tc_fence_after();
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t rr[32];
            tmem_ld32(tO + c * 32, rr);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tmem_st32(tO + c * 32, rr);
          }
        }
#pragma unroll
        for (int c = 0; c < BN / 64; ++c) tmem_st32(tP + c * 32, pk[c]);
        if (j == 0 && pend_out) {
          uint32_t ob[D / 32][32], ow[D / 2];
          read_o<D>(tO, ob);
          pack_o<T, D>(ob, pend_inv, ow);
          store_o<T, D>(ow, pend_orow);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        ++pn;
        pend_out = false;
      }
      if (!ok) break;
      // O / l for valid rows, zeros for var-len padding rows; rows past S not stored
      pend_out = true;
      pend_orow = row < p.S ? orow : nullptr;
      const bool has_keys = l > 0.f && row < it.seq_len;
      pend_inv = has_keys ? 1.f / l : 0.f;
      // LSE in natural log (final once the last tile is exponentiated): the
      // running max is kept in log2 units and P = 2^(x - m)
      if (LSE && row < p.S)
        p.lse[(int64_t)it.b * p.lse_sb + (int64_t)hq * p.lse_sh + row] =
            has_keys ? (m_use + __log2f(l)) * kLn2 : -INFINITY;
    }
    if (ok && pend_out && wait(&pv_done[t], pc & 1)) {
      ++pc;
      tc_fence_after();
      uint32_t ob[D / 32][32], ow[D / 2];
      read_o<D>(tO, ob);
      pack_o<T, D>(ob, pend_inv, ow);
      store_o<T, D>(ow, pend_orow);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// -------------------------------------------------------------------------
// host: tensor maps through the driver entry point (no -lcuda)
// -------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

// 4-D map over [B][H][S][D] (element strides sb, sh, ss; dim stride 1), box 64 x 128
int make_map(CUtensorMap* m, const void* base, int dtype, int B, int H, int S, int D, int64_t sb, int64_t sh,
             int64_t ss, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(AKT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, dtype == AKT_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AKT_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return AKT_OK;
}

// SM count of the current device, cached per device (host threads may race on
// the first call; each computes the same value)
int sm_count() {
  static std::atomic<int> counts[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = counts[dev].load(std::memory_order_relaxed);
  if (!n) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T, int D, bool LSE, bool SCHED>
int launch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const PrefillParams& p,
                   cudaStream_t st) {
  auto kern = prefill_fwd_kernel<T, D, LSE, SCHED>;
  const int smem = (int)(SCHED ? Cfg<D>::SMEM_SCHED : Cfg<D>::SMEM);
  // the register split in the kernel is only valid at the compiled count
  // (read once per instantiation; the static's initialisation is thread-safe)
  static const int regs = [&] {
    cudaFuncAttributes fa;
    return cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : 0;
  }();
  if (regs != kLaunchRegs)
    return set_error(AKT_ERR_CUDA, "prefill kernel compiled with " + std::to_string(regs) + " registers, expected " +
                                       std::to_string(kLaunchRegs));
  cudaError_t e = ensure_smem_limit<prefill_fwd_kernel<T, D, LSE, SCHED>>((size_t)smem);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  const int grid = std::min(p.n_items, sm_count());  // persistent: one CTA per SM
  {
    ProfileScope prof(st);
    kern<<<grid, kThreads, smem, st>>>(mq, mk, mv, p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("prefill launch: ") + cudaGetErrorString(e));
  return AKT_OK;
}

// the kernel variant for the output (LSE or not) and the work order
template <typename T, int D>
int dispatch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const PrefillParams& p,
                     bool lse, bool sched, cudaStream_t st) {
  if (lse)
    return sched ? launch_prefill<T, D, true, true>(mq, mk, mv, p, st) : launch_prefill<T, D, true, false>(mq, mk, mv, p, st);
  return sched ? launch_prefill<T, D, false, true>(mq, mk, mv, p, st) : launch_prefill<T, D, false, false>(mq, mk, mv, p, st);
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

cudaError_t prefill_status_read(unsigned int* v) { return cudaMemcpyFromSymbol(v, g_device_status_local, sizeof(*v)); }

cudaError_t prefill_status_clear() {
  const unsigned int z = 0;
  return cudaMemcpyToSymbol(g_device_status_local, &z, sizeof(z));
}

}  // namespace akt

using namespace akt;

static int prefill_entry(const akt_prefill_args* a, float* lse, int64_t lse_sb, int64_t lse_sh, void* stream) {
  if (!a) return set_error(AKT_ERR_INVALID, "null args");
  if (a->batch < 0 || a->num_qo_heads <= 0 || a->num_kv_heads <= 0 || a->seq_len < 0)
    return set_error(AKT_ERR_INVALID, "sizes must be non-negative");
  if (a->num_qo_heads % a->num_kv_heads) return set_error(AKT_ERR_INVALID, "num_qo_heads must be a multiple of num_kv_heads");
  if (a->head_dim != 64 && a->head_dim != 128) return set_error(AKT_ERR_UNSUPPORTED, "prefill: head_dim must be 64 or 128");
  if (a->dtype != AKT_FLOAT16 && a->dtype != AKT_BFLOAT16) return set_error(AKT_ERR_INVALID, "dtype");
  if (a->q_stride_dim != 1 || a->k_stride_dim != 1 || a->v_stride_dim != 1 || a->out_stride_dim != 1)
    return set_error(AKT_ERR_UNSUPPORTED, "prefill: unit dim stride required");
  const int64_t strides[] = {a->q_stride_batch, a->q_stride_head, a->q_stride_token, a->k_stride_batch,
                             a->k_stride_head,  a->k_stride_token, a->v_stride_batch, a->v_stride_head,
                             a->v_stride_token, a->out_stride_batch, a->out_stride_head, a->out_stride_token};
  for (int64_t s : strides)
    if (s % 8) return set_error(AKT_ERR_UNSUPPORTED, "prefill: strides must be multiples of 16 bytes");
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->out))
    return set_error(AKT_ERR_UNSUPPORTED, "prefill: 16-byte alignment required");
  if (!(a->softmax_scale > 0.f) || a->softmax_scale == INFINITY)
    return set_error(AKT_ERR_UNSUPPORTED, "prefill: softmax_scale must be positive and finite");
  if (a->batch == 0 || a->seq_len == 0) return AKT_OK;
  const int bn = a->head_dim == 64 ? Cfg<64>::BN : Cfg<128>::BN;
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, a->q, a->dtype, a->batch, a->num_qo_heads, a->seq_len, a->head_dim, a->q_stride_batch,
                    a->q_stride_head, a->q_stride_token, BM);
  if (!rc) rc = make_map(&mk, a->k, a->dtype, a->batch, a->num_kv_heads, a->seq_len, a->head_dim, a->k_stride_batch,
                         a->k_stride_head, a->k_stride_token, bn);
  if (!rc) rc = make_map(&mv, a->v, a->dtype, a->batch, a->num_kv_heads, a->seq_len, a->head_dim, a->v_stride_batch,
                         a->v_stride_head, a->v_stride_token, bn);
  if (rc) return rc;
  PrefillParams p{};
  p.o = a->out;
  p.o_sb = a->out_stride_batch; p.o_sh = a->out_stride_head; p.o_ss = a->out_stride_token;
  p.varlen = a->varlen;
  p.B = a->batch; p.Hq = a->num_qo_heads; p.Hkv = a->num_kv_heads; p.S = a->seq_len;
  p.group = p.Hq / p.Hkv;
  p.n_q_tiles = (a->seq_len + BM - 1) / BM;
  p.pair_heads = p.group % 2 == 0 ? 1 : 0;
  const int64_t items = p.pair_heads ? (int64_t)p.n_q_tiles * p.B * (p.Hq / 2)
                                     : (int64_t)((p.n_q_tiles + 1) / 2) * p.B * p.Hq;
  if (items > INT32_MAX) return set_error(AKT_ERR_UNSUPPORTED, "prefill: too many query tiles");
  p.n_items = (int)items;
  p.causal = a->causal ? 1 : 0;
  p.scale_log2 = a->softmax_scale * kLog2e;
  p.lse = lse;
  p.lse_sb = lse_sb;
  p.lse_sh = lse_sh;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // var-len work order from the lengths when the table holds the batch (any
  // other call keeps the plain order)
  const int levels = p.pair_heads ? p.n_q_tiles : (p.n_q_tiles + 1) / 2;
  const bool sched = p.varlen && p.B <= kSchedMaxB && levels <= kSchedMaxTiles;
  if (a->dtype == AKT_FLOAT16)
    return a->head_dim == 64 ? dispatch_prefill<__half, 64>(mq, mk, mv, p, lse != nullptr, sched, st)
                             : dispatch_prefill<__half, 128>(mq, mk, mv, p, lse != nullptr, sched, st);
  return a->head_dim == 64 ? dispatch_prefill<__nv_bfloat16, 64>(mq, mk, mv, p, lse != nullptr, sched, st)
                           : dispatch_prefill<__nv_bfloat16, 128>(mq, mk, mv, p, lse != nullptr, sched, st);
}

extern "C" int akt_prefill(const akt_prefill_args* a, void* stream) { return prefill_entry(a, nullptr, 0, 0, stream); }

extern "C" int akt_prefill_with_lse(const akt_prefill_args* a, float* lse, int64_t lse_stride_batch,
                                    int64_t lse_stride_head, void* stream) {
  if (!lse) return set_error(AKT_ERR_INVALID, "prefill: lse output required");
  return prefill_entry(a, lse, lse_stride_batch, lse_stride_head, stream);
}
