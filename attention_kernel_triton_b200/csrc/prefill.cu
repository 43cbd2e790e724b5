// Causal / non-causal GQA prefill (flash-attention forward) for sm_100a on the
// 5th-generation tensor cores (tcgen05 + TMEM), with padded var-len support.
//
// Replaces the Triton kernels of prefill_flash_attention.py:109-335 and
// prefill_flash_attention_var_len_padding.py:109-341.  Same math:
// O = softmax(Q K^T * s [+ top-left causal mask]) V with GQA kv head h / G,
// fp32 accumulation, P rounded to the input dtype before P.V (PF:94); the
// var-len variant skips query rows past each sequence's length (PV:186-187)
// and masks no keys (the reference does not either).
//
// One CTA = one 128-row query tile of one (batch, head).  Warp roles:
//   warps 0-3  softmax warpgroup: thread t owns query row t = TMEM lane t;
//              reads S with tcgen05.ld, writes P (input dtype) to shared
//              memory in the 128B-swizzled K-major layout, rescales O in
//              TMEM when its running max moves, and runs the epilogue.
//   warp 4     TMA producer: Q once, then K_j and V_j into a ring of stages.
//   warp 5     TMEM allocator and single-thread MMA issuer:
//              S_j = Q K_j^T  (M=128, N=128, K=D)   into TMEM S[j%2]
//              O  += P_j V_j  (M=128, N=D,  K=128)  into TMEM O
// The running max used for exponentiation only moves when the row max grows
// by more than 8 (log2 units), so O is rescaled rarely (P <= 2^8 stays exact
// enough in fp16/bf16 relative terms; the final O/l is unchanged).
#include "common.cuh"
#include "profile.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

namespace akt {

int set_error(int code, const std::string& msg);

namespace {

constexpr int BM = 128;            // query rows per CTA
constexpr int kThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__host__ __device__ constexpr int pow2_at_least(int x) {
  int v = 32;
  while (v < x) v *= 2;
  return v;
}

// Tile configuration per (head_dim D, keys per tile BN).  TMEM holds S
// (NSB buffers of BN fp32 columns) and O (D columns); shared memory holds Q,
// a two-stage K/V ring and one P tile.  Smaller footprints let more CTAs (and
// so more softmax warpgroups) share an SM:
//   D=64,  BN=64 : TMEM 128 cols,  64 KB smem -> 3 CTAs/SM
//   D=64,  BN=128: TMEM 256 cols, 112 KB smem -> 2 CTAs/SM
//   D=128, BN=64 : TMEM 256 cols, 112 KB smem -> 2 CTAs/SM
//   D=128, BN=128: TMEM 512 cols (S double-buffered), 192 KB -> 1 CTA/SM
template <int D, int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int DB = D / 64;                       // 64-element (128 B) swizzle blocks per row
  static constexpr int NSB = (D == 128 && BN == 128) ? 2 : 1;
  static constexpr int COL_O = NSB * BN;
  static constexpr int TMEM_COLS = pow2_at_least(COL_O + D);
  // K and V rings are separate: a K stage is released when its S MMA is done,
  // a V stage when its P.V MMA is done, so K loads run further ahead.
  static constexpr int NSK = (D == 64 && BN == 64) ? 3 : 2;
  static constexpr int NSV = 2;
  static constexpr int NP = 1;                            // P buffers
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;        // one K or V tile
  static constexpr uint32_t P_BYTES = BM * BN * 2;
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + NSK * KV_BYTES;
  static constexpr uint32_t OFF_P = OFF_V + NSV * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_P + NP * P_BYTES;
  static constexpr uint32_t SMEM = OFF_BAR + 256;         // + barriers (base is 1024-aligned)
  static constexpr int CTAS_PER_SM = (SMEM + 1024) * 3 <= 228 * 1024 && TMEM_COLS * 3 <= 512 ? 3
                                     : (SMEM + 1024) * 2 <= 228 * 1024 && TMEM_COLS * 2 <= 512 ? 2 : 1;
};

struct PrefillParams {
  void* o;
  int64_t o_sb, o_sh, o_ss;  // element strides (dim stride 1)
  const int32_t* varlen;     // [B] or null
  int B, Hq, Hkv, S, group;
  int n_q_tiles;
  int causal;
  float scale_log2;
};

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

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
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

// one lane of a converged warp (the issuing lane for MMA / TMA / commit)
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "@px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

template <typename T>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
  return Elem<T>::pack2(a, b);
}

// -------------------------------------------------------------------------
// kernel
// -------------------------------------------------------------------------
template <typename T, int D, int BN>
__global__ void __launch_bounds__(kThreads, (Cfg<D, BN>::CTAS_PER_SM))
    prefill_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const PrefillParams p) {
  using C = Cfg<D, BN>;
  constexpr int fmt = std::is_same<T, __half>::value ? 0 : 1;
  constexpr uint32_t IDESC_S = idesc_f16(fmt, BM, BN, 0);
  constexpr uint32_t IDESC_PV = idesc_f16(fmt, BM, D, 1);

  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023u) {  // swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_status(kStatusWaitTimeout);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                   // [NSK]
  uint64_t* k_empty = k_full + C::NSK;           // [NSK]
  uint64_t* v_full = k_empty + C::NSK;           // [NSV]
  uint64_t* v_empty = v_full + C::NSV;           // [NSV]
  uint64_t* s_full = v_empty + C::NSV;           // [NSB]
  uint64_t* s_empty = s_full + C::NSB;           // [NSB]
  uint64_t* p_full = s_empty + C::NSB;           // [NP]
  uint64_t* p_empty = p_full + C::NP;            // [NP]
  uint64_t* o_done = p_empty + C::NP;            // 1
  uint64_t* mma_idle = o_done + 1;               // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_idle + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_tile = p.n_q_tiles - 1 - (int)blockIdx.x;  // heaviest causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = q_tile * BM;
  const int seq_len = p.varlen ? min(max(p.varlen[b], 0), p.S) : p.S;

  // ---- tile entirely past the sequence (var-len padding): zeros, no MMA
  if (q0 >= seq_len) {
    T* o = static_cast<T*>(p.o) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh;
    for (int e = threadIdx.x; e < BM * (D / 8); e += kThreads) {
      const int r = q0 + e / (D / 8), c = (e % (D / 8)) * 8;
      if (r < p.S) *reinterpret_cast<uint4*>(o + (int64_t)r * p.o_ss + c) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int last_key = p.causal ? min(q0 + BM, seq_len) - 1 : p.S - 1;  // causal: rows past seq_len are zeroed
  const int n_kv = last_key / BN + 1;
  const int kvh = h / p.group;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NSK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::NSV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < C::NSB; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    for (int s = 0; s < C::NP; ++s) {
      mbar_init(&p_full[s], 4);
      mbar_init(&p_empty[s], 1);
    }
    mbar_init(o_done, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(bar, parity)) return true;
    *abort_flag = 1;
    return false;
  };
  // warp-uniform variant for the warp that issues MMAs in lockstep
  auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, wait(bar, parity)) != 0;
  };

  if (warp == 4) {
    // ========================= TMA producers =========================
    // lane 0: Q, then the K ring; lane 1: the V ring (independent waits)
    if (lane == 0) {
      unsigned char* sQ = smem + C::OFF_Q;
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int db = 0; db < C::DB; ++db) tma_load_4d(sQ + db * BM * 128, &tmQ, db * 64, q0, h, b, q_full);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::NSK;
        if (j >= C::NSK && !wait(&k_empty[st], ((j / C::NSK) - 1) & 1)) break;
        unsigned char* sK = smem + C::OFF_K + st * C::KV_BYTES;
        mbar_arrive_expect_tx(&k_full[st], C::KV_BYTES);
#pragma unroll
        for (int db = 0; db < C::DB; ++db) tma_load_4d(sK + db * BN * 128, &tmK, db * 64, j * BN, kvh, b, &k_full[st]);
        issued = j + 1;
      }
      if (*abort_flag) {  // drain loads still in flight into this CTA's shared memory
        mbar_wait(q_full, 0);
        for (int j = max(0, issued - C::NSK); j < issued; ++j) mbar_wait(&k_full[j % C::NSK], (j / C::NSK) & 1);
      }
    } else if (lane == 1) {
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::NSV;
        if (j >= C::NSV && !wait(&v_empty[st], ((j / C::NSV) - 1) & 1)) break;
        unsigned char* sV = smem + C::OFF_V + st * C::KV_BYTES;
        mbar_arrive_expect_tx(&v_full[st], C::KV_BYTES);
#pragma unroll
        for (int db = 0; db < C::DB; ++db) tma_load_4d(sV + db * BN * 128, &tmV, db * 64, j * BN, kvh, b, &v_full[st]);
        issued = j + 1;
      }
      if (*abort_flag) {
        for (int j = max(0, issued - C::NSV); j < issued; ++j) mbar_wait(&v_full[j % C::NSV], (j / C::NSV) & 1);
      }
    }
  } else if (warp == 5) {
    // ========================= MMA issuer =========================
    // The whole warp runs the loop (descriptors stay warp-uniform); one
    // elected lane issues each MMA and commit.
    const uint32_t sQ = smem_u32(smem + C::OFF_Q);
    bool ok = wwait(q_full, 0);
    tc_fence_after();
    for (int j = 0; ok && j <= n_kv; ++j) {
      if (j < n_kv) {
        const int st = j % C::NSK, sb = j % C::NSB;
        if (!wwait(&k_full[st], (j / C::NSK) & 1)) break;
        if (j >= C::NSB && !wwait(&s_empty[sb], ((j / C::NSB) - 1) & 1)) break;
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + C::OFF_K + st * C::KV_BYTES);
        const bool leader = elect_one();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * (BM * 128) + (k & 3) * 32;
          const uint32_t offk = (k >> 2) * (BN * 128) + (k & 3) * 32;
          const uint64_t da = desc_sw128(sQ + off, 16, 1024), db = desc_sw128(sK + offk, 16, 1024);
          if (leader) mma_f16(tmem + sb * BN, da, db, IDESC_S, k > 0);
        }
        if (leader) {
          mma_commit(&s_full[sb]);
          mma_commit(&k_empty[st]);
        }
        __syncwarp();
      }
      if (j >= 1) {
        const int i = j - 1, pb = i % C::NP, st = i % C::NSV;
        if (!wwait(&p_full[pb], (i / C::NP) & 1)) break;
        if (!wwait(&v_full[st], (i / C::NSV) & 1)) break;
        tc_fence_after();
        const uint32_t sP = smem_u32(smem + C::OFF_P + pb * C::P_BYTES);
        const uint32_t sV = smem_u32(smem + C::OFF_V + st * C::KV_BYTES);
        const bool leader = elect_one();
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint32_t offp = (k >> 2) * (BM * 128) + (k & 3) * 32;
          const uint64_t da = desc_sw128(sP + offp, 16, 1024), db = desc_sw128(sV + k * 2048, BN * 128, 1024);
          if (leader) mma_f16(tmem + C::COL_O, da, db, IDESC_PV, (i > 0 || k > 0) ? 1u : 0u);
        }
        if (leader) {
          mma_commit(o_done);
          mma_commit(&p_empty[pb]);
          mma_commit(&v_empty[st]);
        }
        __syncwarp();
      }
    }
    // every MMA issued by this warp has finished before the CTA can exit
    if (elect_one()) mma_commit(mma_idle);
    __syncwarp();
    mbar_wait(mma_idle, 0);
  } else {
    // ========================= softmax warpgroup =========================
    const int t = threadIdx.x;  // 0..127: row t of the tile, TMEM lane t
    const int row = q0 + t;
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    float m_use = -INFINITY, l = 0.f;
    int pv_seen = 0;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j % C::NSB, pb = j % C::NP;
      if (!wait(&s_full[sb], (j / C::NSB) & 1)) { ok = false; break; }
      tc_fence_after();
      float x[BN];
      {
        uint32_t r[BN / 32][32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tmem + lane_addr + sb * BN + c * 32, r[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(r[c][e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      // masks only where a key tile reaches past the tile's first row (causal
      // diagonal) or past S
      if ((p.causal && (j + 1) * BN - 1 > q0) || (j + 1) * BN > p.S) {
        const int lim = min(p.causal ? row : p.S - 1, p.S - 1) - j * BN;  // last visible column
#pragma unroll
        for (int c = 0; c < BN; ++c) x[c] = c > lim ? -INFINITY : x[c];
      }
      // row max of the raw scores (scale > 0), 8 independent chains
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = x[e];
#pragma unroll
      for (int c = 8; c < BN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], x[c]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * p.scale_log2;
      const float m_new = fmaxf(m_use, mx);
      const bool need = m_new > m_use + kRescaleThreshold || (m_use == -INFINITY && m_new != -INFINITY);
      float alpha = 1.f;
      if (need) {
        alpha = fast_exp2(m_use - m_new);
        m_use = m_new;
      }
      const float m_sub = m_use == -INFINITY ? 0.f : m_use;
      // P = 2^(s*scale - m) in the input dtype, packed in registers first so the
      // exponentials do not wait for the previous P.V to release the P tile
      float rs8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) rs8[e] = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int ch = 0; ch < BN / 8; ++ch) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = fast_exp2(fmaf(x[ch * 8 + e], p.scale_log2, -m_sub));
          rs8[e] += pv[e];
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) pk[ch * 4 + e] = pack_p<T>(pv[2 * e], pv[2 * e + 1]);
      }
      if (j >= C::NP && !wait(&p_empty[pb], ((j / C::NP) - 1) & 1)) { ok = false; break; }
      unsigned char* sP = smem + C::OFF_P + pb * C::P_BYTES;
#pragma unroll
      for (int ch = 0; ch < BN / 8; ++ch) {
        const int kb = ch >> 3, cin = ch & 7;
        *reinterpret_cast<uint4*>(sP + kb * (BM * 128) + t * 128 + ((cin ^ (t & 7)) << 4)) =
            make_uint4(pk[ch * 4 + 0], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
      }
      const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      l = l * alpha + rs;
      // O must see PV_{j-1} finished before it is rescaled or before PV_j is queued
      if (j >= 1) {
        while (pv_seen < j) {
          if (!wait(o_done, pv_seen & 1)) { ok = false; break; }
          ++pv_seen;
        }
        if (!ok) break;
        if (__any_sync(0xffffffffu, need)) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem + lane_addr + C::COL_O + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st32(tmem + lane_addr + C::COL_O + c * 32, r);
          }
          tmem_wait_st();
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);
    }
    // ---- epilogue: O / l for valid rows, zeros for var-len padding rows
    if (ok) {
      while (pv_seen < n_kv) {
        if (!wait(o_done, pv_seen & 1)) { ok = false; break; }
        ++pv_seen;
      }
    }
    T* orow = static_cast<T*>(p.o) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)row * p.o_ss;
    const float inv = (ok && l > 0.f && row < seq_len) ? 1.f / l : 0.f;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_addr + C::COL_O + c * 32, r);
      tmem_wait_ld();
      if (row < p.S) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = Elem<T>::pack2(__uint_as_float(r[e + 0]) * inv, __uint_as_float(r[e + 1]) * inv);
          w.y = Elem<T>::pack2(__uint_as_float(r[e + 2]) * inv, __uint_as_float(r[e + 3]) * inv);
          w.z = Elem<T>::pack2(__uint_as_float(r[e + 4]) * inv, __uint_as_float(r[e + 5]) * inv);
          w.w = Elem<T>::pack2(__uint_as_float(r[e + 6]) * inv, __uint_as_float(r[e + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + e) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// -------------------------------------------------------------------------
// host: tensor maps through the driver entry point (no -lcuda)
// -------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

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

template <typename T, int D, int BN>
int launch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const PrefillParams& p,
                   cudaStream_t st) {
  auto kern = prefill_fwd_kernel<T, D, BN>;
  const int smem = (int)Cfg<D, BN>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  dim3 grid(p.n_q_tiles, p.Hq, p.B);
  {
    ProfileScope prof(st);
    kern<<<grid, kThreads, smem, st>>>(mq, mk, mv, p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, std::string("prefill launch: ") + cudaGetErrorString(e));
  return AKT_OK;
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// keys per tile: AKT_PREFILL_BN (64 or 128) overrides the default, read once
int prefill_key_tile(int D) {
  static int forced = -1;
  if (forced < 0) {
    const char* v = getenv("AKT_PREFILL_BN");
    forced = v ? atoi(v) : 0;
    if (forced != 64 && forced != 128) forced = 0;
  }
  if (forced) return forced;
  return D == 64 ? 64 : 128;
}

}  // namespace
}  // namespace akt

using namespace akt;

extern "C" int akt_prefill(const akt_prefill_args* a, void* stream) {
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
  const int bn = prefill_key_tile(a->head_dim);
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
  p.causal = a->causal ? 1 : 0;
  p.scale_log2 = a->softmax_scale * kLog2e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == AKT_FLOAT16) {
    if (a->head_dim == 64)
      return bn == 64 ? launch_prefill<__half, 64, 64>(mq, mk, mv, p, st) : launch_prefill<__half, 64, 128>(mq, mk, mv, p, st);
    return bn == 64 ? launch_prefill<__half, 128, 64>(mq, mk, mv, p, st) : launch_prefill<__half, 128, 128>(mq, mk, mv, p, st);
  }
  if (a->head_dim == 64)
    return bn == 64 ? launch_prefill<__nv_bfloat16, 64, 64>(mq, mk, mv, p, st)
                    : launch_prefill<__nv_bfloat16, 64, 128>(mq, mk, mv, p, st);
  return bn == 64 ? launch_prefill<__nv_bfloat16, 128, 64>(mq, mk, mv, p, st)
                  : launch_prefill<__nv_bfloat16, 128, 128>(mq, mk, mv, p, st);
}
