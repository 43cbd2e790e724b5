// Per-warp decode core on the tensor cores (warp-level mma.sync): one query
// row per head for up to 8 heads that share a K/V stream, 16 keys per step.
//
// The reference's decode loop is two dots per key block with fp32
// accumulation, P rounded to the input type before P.V (DP:39-57:
// tl.dot(q, k), exp, P.to(float16), tl.dot(P, V, acc)).  Per step of 16 keys
// this warp computes
//   S^T[16 keys x 8 heads]  = K[16 x D] . q^T[D x 8]        (D/16 MMAs m16n8k16)
//   O^T[D x 8 heads]       += V^T[D x 16] . P^T[16 x 8]      (D/16 MMAs)
// Heads past G are zero columns of q^T.  With keys as the M dimension, the
// S^T accumulator and the O^T accumulator give a lane the same two heads
// (columns 2*(lane%4) and +1), so the running max, the sum and the rescale of
// O stay in the lane; the only exchange is the max over the step's keys
// (three shuffles).  P^T reaches the B-operand layout by one register
// transpose per 8 keys (movmatrix).  Scores are the fp32 dot times
// softmax_scale*log2(e), exponentials exp2 (the log2 domain of the CUDA-core
// decode), P rounded to the input type as in the reference.
//
// Shared-memory tile layout (what a TMA tensor-map load with a 128-byte swizzle
// writes): per 64-column half of D, TT rows of 128 bytes; the 16-byte chunk c
// of row t sits at chunk c ^ (t % 8).  Each half starts on a 1024-byte
// boundary.  ldmatrix then reads 8 rows of one logical chunk from 8 distinct
// chunks of a 128-byte line: no bank conflicts.
#pragma once

#include "common.cuh"

namespace akt {

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
struct MmaOp;

template <>
struct MmaOp<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

template <>
struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

template <typename T, int D, int G>
struct WarpMma {
  static_assert(D % 64 == 0 && D <= 256, "head_dim");
  static_assert(G >= 1 && G <= 8, "heads per warp");
  static constexpr int KS = D / 16;  // k-steps of q.k = 16-row tiles of O^T
  using E = Elem<T>;

  uint32_t qb[KS][2];  // q^T B fragments per k-step
  float o[KS][4];      // O^T accumulators: dims 16*i + lane/4 (+8), heads hA, hB
  float mA, mB;        // running max (log2 units) of heads hA = 2*(lane%4), hB = hA + 1
  float lA, lB;        // this lane's part of the sums of p (its two keys per step)
  int lane;

  __device__ __forceinline__ void init(int lane_) {
    lane = lane_;
    mA = mB = -INFINITY;
    lA = lB = 0.f;
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }

  // q of head h at q0 + h * q_sh (unit dim stride, 4-byte aligned); heads
  // G..7 are zero columns
  __device__ __forceinline__ void load_q(const T* q0, int64_t q_sh) {
    const int h = lane >> 2, c = 2 * (lane & 3);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      if (h < G) {
        const T* r = q0 + (int64_t)h * q_sh + 16 * ks + c;
        qb[ks][0] = *reinterpret_cast<const uint32_t*>(r);
        qb[ks][1] = *reinterpret_cast<const uint32_t*>(r + 8);
      } else {
        qb[ks][0] = qb[ks][1] = 0u;
      }
    }
  }

  // One step over keys [row0, row0 + 16) of a K/V tile (shared addresses of
  // the K and V tiles, half_bytes = bytes per 64-column half).  Keys at or
  // past row0 + ns are masked; their V rows must be finite.  row0 is a
  // multiple of 16.  sc = softmax_scale * log2(e).
  __device__ __forceinline__ void step(uint32_t kbase, uint32_t vbase, uint32_t half_bytes, int row0, int ns,
                                       float sc) {
    const int lr = lane & 7;
    // ---- S^T = K . q^T: ldmatrix matrices (keys 0-7 | 8-15) x (chunk c | c+1)
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int kt = row0 + lr + ((lane >> 3) & 1) * 8;
      const uint32_t krow = kbase + (uint32_t)kt * 128u;
      const int cadd = lane >> 4;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int c = ((ks & 3) << 1) + cadd;
        uint32_t a[4];
        ldsm_x4(a, krow + (uint32_t)(ks >> 2) * half_bytes + (uint32_t)((c ^ lr) << 4));
        MmaOp<T>::run(s, a, qb[ks][0], qb[ks][1]);
      }
    }
    // ---- online softmax (keys g and g + 8 of this step; heads hA, hB)
    const int g = lane >> 2;
    const bool va = g < ns, vb = g + 8 < ns;
    const float s0 = va ? s[0] * sc : -INFINITY, s1 = va ? s[1] * sc : -INFINITY;
    const float s2 = vb ? s[2] * sc : -INFINITY, s3 = vb ? s[3] * sc : -INFINITY;
    float tA = fmaxf(s0, s2), tB = fmaxf(s1, s3);
#pragma unroll
    for (int x = 4; x <= 16; x <<= 1) {
      tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, x));
      tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, x));
    }
    // ns >= 1, so every head has a finite score in this step
    const float nA = fmaxf(mA, tA), nB = fmaxf(mB, tB);
    const float p0 = fast_exp2(s0 - nA), p1 = fast_exp2(s1 - nB);
    const float p2 = fast_exp2(s2 - nA), p3 = fast_exp2(s3 - nB);
    if (__any_sync(0xffffffffu, (nA != mA) | (nB != mB))) {
      const float aA = fast_exp2(mA - nA), aB = fast_exp2(mB - nB);  // 0 on the first step
      lA *= aA;
      lB *= aB;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        o[i][0] *= aA; o[i][1] *= aB;
        o[i][2] *= aA; o[i][3] *= aB;
      }
      mA = nA;
      mB = nB;
    }
    lA += p0 + p2;
    lB += p1 + p3;
    // P^T B fragments: rows of the 8x8 blocks are keys, columns heads; the
    // transpose gives each lane keys 2*(lane%4), +1 of head lane/4
    const uint32_t b0 = movmatrix_trans(E::pack2(p0, p1));
    const uint32_t b1 = movmatrix_trans(E::pack2(p2, p3));
    // ---- O^T += V^T . P^T: ldmatrix.trans matrices (dims c | c+1) x (keys 0-7 | 8-15)
    {
      const int vt = row0 + lr + (lane >> 4) * 8;
      const uint32_t vrow = vbase + (uint32_t)vt * 128u;
      const int cadd = (lane >> 3) & 1;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        const int c = ((i & 3) << 1) + cadd;
        uint32_t a[4];
        ldsm_x4_trans(a, vrow + (uint32_t)(i >> 2) * half_bytes + (uint32_t)((c ^ lr) << 4));
        MmaOp<T>::run(o[i], a, b0, b1);
      }
    }
  }

  // Write this warp's state to the CTA combine buffers (index w), in the
  // layout of the CUDA-core core's stash: m and l per head, O per (head, dim).
  __device__ __forceinline__ void stash(float* comb_m, float* comb_l, float* comb_o, int w, bool alive) {
#pragma unroll
    for (int x = 4; x <= 16; x <<= 1) {
      lA += __shfl_xor_sync(0xffffffffu, lA, x);
      lB += __shfl_xor_sync(0xffffffffu, lB, x);
    }
    const int hA = 2 * (lane & 3), hB = hA + 1, g = lane >> 2;
    if (lane < 4) {
      if (hA < G) {
        comb_m[w * G + hA] = alive ? mA : -INFINITY;
        comb_l[w * G + hA] = alive ? lA : 0.f;
      }
      if (hB < G) {
        comb_m[w * G + hB] = alive ? mB : -INFINITY;
        comb_l[w * G + hB] = alive ? lB : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      const int d = 16 * i + g;
      if (hA < G) {
        comb_o[(w * G + hA) * D + d] = alive ? o[i][0] : 0.f;
        comb_o[(w * G + hA) * D + d + 8] = alive ? o[i][2] : 0.f;
      }
      if (hB < G) {
        comb_o[(w * G + hB) * D + d] = alive ? o[i][1] : 0.f;
        comb_o[(w * G + hB) * D + d + 8] = alive ? o[i][3] : 0.f;
      }
    }
  }
};

}  // namespace akt
