// Per-warp attention core shared by the decode kernels (dense, paged, sparse,
// MagicPIG): one query row per head for G heads that share a K/V stream.
//
// Lane layout for q.k: 8 lanes per K row (4 rows per warp pass); lane li of
// a row group owns the 16-byte chunks li, li+8, ... of the row.  After the
// partial dot products, an 8-lane reduce-scatter leaves each lane the full
// score of one (row, head): head my_head = li / (8/G).
// Layout for P.V: lane owns D/32 consecutive output dims of every head.
// Online softmax in the log2 domain (exp2), fp32 state, per warp.
#pragma once

#include "common.cuh"

namespace akt {

constexpr int kRowsPerSubTile = 16;  // rows per online-softmax step

template <typename T, int D, int G, bool KNORM>
struct WarpAttn {
  static_assert(D % 64 == 0 && D <= 256, "head_dim");
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "group tile");
  static constexpr int CH = D / 64;   // 16-byte chunks per lane per row
  static constexpr int DPL = D / 32;  // output dims per lane
  static constexpr int LPH = 8 / G;   // lanes holding the same (row, head) score
  using E = Elem<T>;

  float2 qf[G][CH][4];
  float m_own;  // running max (log2 units) of head my_head
  float l_own;  // partial sum of p over this lane's rows, head my_head
  float2 o[G][DPL / 2];
  int lane, tg, li, my_head;

  __device__ __forceinline__ void init(int lane_) {
    lane = lane_;
    tg = lane >> 3;
    li = lane & 7;
    my_head = li / LPH;
    m_own = -INFINITY;
    l_own = 0.f;
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int j = 0; j < DPL / 2; ++j) o[h][j] = make_float2(0.f, 0.f);
  }

  // q of head h at q0 + h * q_sh (unit dim stride, 16-byte aligned), times mult
  __device__ __forceinline__ void load_q(const T* q0, int64_t q_sh, float mult) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const T* qh = q0 + (int64_t)h * q_sh;
#pragma unroll
      for (int cc = 0; cc < CH; ++cc) {
        const uint4 raw = *reinterpret_cast<const uint4*>(qh + (li + 8 * cc) * 8);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = E::to_float2(w[j]);
          qf[h][cc][j] = make_float2(f.x * mult, f.y * mult);
        }
      }
    }
  }

  // |q_h|^2 of head my_head (fp32 sum of squares of the loaded q, mult=1)
  // (each head's partial sums are reduced over the 8 lanes of the row group
  // before the lane picks its own head)
  __device__ __forceinline__ float q_norm2_my_head() const {
    float s = 0.f;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float t = 0.f;
#pragma unroll
      for (int cc = 0; cc < CH; ++cc)
#pragma unroll
        for (int j = 0; j < 4; ++j) t += qf[h][cc][j].x * qf[h][cc][j].x + qf[h][cc][j].y * qf[h][cc][j].y;
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      t += __shfl_xor_sync(0xffffffffu, t, 4);
      if (h == my_head) s = t;
    }
    return s;
  }

  // dot(q_{my_head}, k_row) after the reduce-scatter; |k|^2 if KNORM
  __device__ __forceinline__ float qk_row(const T* row, float& kk) const {
    float2 acc[G];
    float2 acck = make_float2(0.f, 0.f);
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h] = make_float2(0.f, 0.f);
#pragma unroll
    for (int cc = 0; cc < CH; ++cc) {
      const uint4 raw = *reinterpret_cast<const uint4*>(row + (li + 8 * cc) * 8);
      const float2 k[4] = {E::to_float2(raw.x), E::to_float2(raw.y), E::to_float2(raw.z), E::to_float2(raw.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int h = 0; h < G; ++h) acc[h] = ffma2(qf[h][cc][j], k[j], acc[h]);
        if (KNORM) acck = ffma2(k[j], k[j], acck);
      }
    }
    float v[G];
#pragma unroll
    for (int h = 0; h < G; ++h) v[h] = acc[h].x + acc[h].y;
#pragma unroll
    for (int step = 4, cnt = G; step >= 1; step >>= 1) {
      if (cnt > 1) {
        const bool upper = (li & step) != 0;
#pragma unroll
        for (int j = 0; j < cnt / 2; ++j) {
          const float send = upper ? v[j] : v[j + cnt / 2];
          const float keep = upper ? v[j + cnt / 2] : v[j];
          v[j] = keep + __shfl_xor_sync(0xffffffffu, send, step);
        }
        cnt >>= 1;
      } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], step);
      }
    }
    if (KNORM) {
      float s = acck.x + acck.y;
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      kk = s;
    } else {
      kk = 0.f;
    }
    return v[0];
  }

  // One step over rows [row0, row0 + 16) of a K/V tile in shared memory.
  // Rows >= row0 + ns, and rows whose bit in valid_bits is clear, are masked
  // (their V rows must be finite: zero-filled or real data).  Rows above
  // row_max are never read.  score(dot, kk, head) maps a raw dot product to
  // a log2-domain score.  pw: this warp's [16][G] float scratch.
  // SHORT: steps may hold fewer than 16 rows (the sparse gather's 8 rows per
  // warp), so four-row passes wholly past ns are skipped, score included.
  template <bool SHORT = false, class ScoreFn>
  __device__ __forceinline__ void step(const T* Ks, const T* Vs, int row0, int ns, int row_max,
                                       uint32_t valid_bits, float* pw, const ScoreFn& score) {
    float sc[kRowsPerSubTile / 4];
#pragma unroll
    for (int pass = 0; pass < kRowsPerSubTile / 4; ++pass) {
      if (SHORT) {
        sc[pass] = -INFINITY;
        if (pass * 4 >= ns) continue;  // warp-uniform
      }
      const int r = pass * 4 + tg;
      const int row = min(row0 + r, row_max);
      float kk;
      const float dot = qk_row(Ks + (size_t)row * D, kk);
      const bool valid = r < ns && ((valid_bits >> r) & 1u);
      if (SHORT) {
        if (valid) sc[pass] = score(dot, kk, my_head);
      } else {
        sc[pass] = valid ? score(dot, kk, my_head) : -INFINITY;
      }
    }
    float mt = sc[0];
#pragma unroll
    for (int j = 1; j < kRowsPerSubTile / 4; ++j) mt = fmaxf(mt, sc[j]);
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
    if (__all_sync(0xffffffffu, mt == -INFINITY)) return;  // nothing valid in this step
    const float m_new = fmaxf(m_own, mt);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;  // a head with no finite score yet
    const float alpha_own = fast_exp2(m_own - m_use);
    float ps = 0.f;
#pragma unroll
    for (int j = 0; j < kRowsPerSubTile / 4; ++j) {
      const float pj = fast_exp2(sc[j] - m_use);
      ps += pj;
      if ((li % LPH) == 0) pw[(j * 4 + tg) * G + my_head] = pj;
    }
    l_own = l_own * alpha_own + ps;
    m_own = m_new;
    float alpha[G];
#pragma unroll
    for (int h = 0; h < G; ++h) alpha[h] = __shfl_sync(0xffffffffu, alpha_own, h * LPH);
    __syncwarp();
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int j = 0; j < DPL / 2; ++j) o[h][j] = fmul2(o[h][j], make_float2(alpha[h], alpha[h]));
    if (ns == kRowsPerSubTile) {
#pragma unroll
      for (int r = 0; r < kRowsPerSubTile; ++r) pv_row(Vs, pw, row0, r);
    } else {
      for (int r = 0; r < ns; ++r) pv_row(Vs, pw, row0, r);
    }
    __syncwarp();
  }

  // o[h] += p[r][h] * V[row0 + r] for this lane's dims
  __device__ __forceinline__ void pv_row(const T* Vs, const float* pw, int row0, int r) {
    {
      float pr[G];
      if constexpr (G % 4 == 0) {
#pragma unroll
        for (int h4 = 0; h4 < G; h4 += 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(pw + r * G + h4);
          pr[h4] = t4.x; pr[h4 + 1] = t4.y; pr[h4 + 2] = t4.z; pr[h4 + 3] = t4.w;
        }
      } else if constexpr (G == 2) {
        const float2 t2 = *reinterpret_cast<const float2*>(pw + r * G);
        pr[0] = t2.x; pr[1] = t2.y;
      } else {
        pr[0] = pw[r];
      }
      const T* vrow = Vs + (size_t)(row0 + r) * D + lane * DPL;
      float2 vf[DPL / 2];
      if constexpr (DPL == 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(vrow);
        vf[0] = E::to_float2(raw.x); vf[1] = E::to_float2(raw.y);
        vf[2] = E::to_float2(raw.z); vf[3] = E::to_float2(raw.w);
      } else if constexpr (DPL == 4) {
        const uint2 raw = *reinterpret_cast<const uint2*>(vrow);
        vf[0] = E::to_float2(raw.x); vf[1] = E::to_float2(raw.y);
      } else {
        vf[0] = E::to_float2(*reinterpret_cast<const uint32_t*>(vrow));
      }
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int j = 0; j < DPL / 2; ++j) o[h][j] = ffma2(make_float2(pr[h], pr[h]), vf[j], o[h][j]);
    }
  }

  // Write this warp's state to the CTA combine buffers (index w).
  __device__ __forceinline__ void stash(float* comb_m, float* comb_l, float* comb_o, int w, bool alive) const {
    float l_tot = l_own;
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 8);
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 16);
    if (lane < 8 && (li % LPH) == 0) {
      comb_m[w * G + my_head] = alive ? m_own : -INFINITY;
      comb_l[w * G + my_head] = alive ? l_tot : 0.f;
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int j = 0; j < DPL / 2; ++j)
        *reinterpret_cast<float2*>(comb_o + (w * G + h) * D + lane * DPL + 2 * j) = o[h][j];
  }
};

// Merge NW warp states for element (h, d): returns normalised value, sets
// lse2 = M + log2(den) (-inf when nothing was attended).
template <int NW, int G, int D>
__device__ __forceinline__ float combine_warps(const float* comb_m, const float* comb_l, const float* comb_o, int h,
                                               int d, float& lse2) {
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < NW; ++w) M = fmaxf(M, comb_m[w * G + h]);
  float den = 0.f, num = 0.f;
  if (M != -INFINITY) {
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float s = fast_exp2(comb_m[w * G + h] - M);
      den += s * comb_l[w * G + h];
      num += s * comb_o[(w * G + h) * D + d];
    }
  }
  lse2 = den > 0.f ? M + log2f(den) : -INFINITY;
  return den > 0.f ? num / den : 0.f;
}

// plain scaled dot-product score (q pre-multiplied by scale*log2(e))
struct ScaledDotScore {
  __device__ __forceinline__ float operator()(float dot, float, int) const { return dot; }
};

}  // namespace akt
