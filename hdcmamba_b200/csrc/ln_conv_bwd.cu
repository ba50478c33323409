// Backward of the fused LayerNorm + causal depthwise conv1d (width 4), sm_100a.
//
// Same formulas as the reference _fused_norm_conv_bwd_kernel (hdcmamba/model.py:74-124)
// and its launch (model.py:148-166), quirks included:
//   dn[t]    = go[t] cw3 + go[t+1] cw2 + go[t+2] cw1 + go[t+3] cw0       (go = 0 past L)
//   xhat[t]  = (x[t] - mean[t]) rstd[t]          (the forward's bf16-stored mean / rstd)
//   dx[t]    = rstd[t] (dn nw - sum(dn nw)/D - xhat sum(dn nw xhat)/D)
//   d_nw     = sum_t dn xhat,  d_nb = sum_t dn,  d_cb = sum_t go[t]
//   d_cw[k]  = sum_t go[t] xhat[t-3+k] nw        (rows t-3+k < 0 contribute nothing, and
//                                                 the norm bias is not part of the term)
// Schedule (HBM-bound: read go, x; write dx):
//   * one CTA walks a contiguous L-segment of one batch row; thread g owns channels
//     [4g, 4g+4), loaded / stored as one 8-byte (bf16) or 16-byte (fp32) vector;
//   * the four grad-output rows t..t+3 and the normalised rows t-3..t of its channels sit in
//     register rings indexed by row mod 4; with segments of a multiple of 4 rows and the row
//     loop unrolled by 4, every ring index is a compile-time constant;
//   * the two row sums of the LayerNorm backward are reduced over the CTA once per 4 rows
//     (warp shuffles, then shared memory; the two halves alternate, one barrier per group);
//   * parameter gradients accumulate in registers per thread and are written per CTA to a
//     workspace, which a second kernel sums over the CTAs in a fixed order (deterministic;
//     the reference adds with fp32 atomics).
#include <algorithm>
#include <type_traits>

#include "tc.cuh"

namespace hdc {

struct LnConvBwdParams {
  const void* go; const void* x; const __nv_bfloat16* mean; const __nv_bfloat16* rstd;
  const void* nw; const void* cw; void* dx; float* part;
  int L, D, seg_len, segs_per_b;
};

template <typename T>
__device__ __forceinline__ void ld4(const T* p, float* f);
template <>
__device__ __forceinline__ void ld4<float>(const float* p, float* f) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
template <>
__device__ __forceinline__ void ld4<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
  f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
}
template <typename T>
__device__ __forceinline__ void st4(T* p, const float* f);
template <>
__device__ __forceinline__ void st4<float>(float* p, const float* f) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
template <>
__device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, const float* f) {
  __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), c = __floats2bfloat162_rn(f[2], f[3]);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&a);
  v.y = *reinterpret_cast<uint32_t*>(&c);
  *reinterpret_cast<uint2*>(p) = v;
}

template <typename T>
__global__ void __launch_bounds__(512) ln_conv_bwd_kernel(LnConvBwdParams p) {
  __shared__ float red[2][4][2][16];  // [half][row of the group][sum][warp]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int seg = blockIdx.x;
  const int b = seg / p.segs_per_b;
  const int l0 = (seg - b * p.segs_per_b) * p.seg_len;
  const int l1 = min(l0 + p.seg_len, p.L);
  const int c0 = tid * 4;
  const bool act = c0 < p.D;
  const int cc = act ? c0 : 0;
  const size_t rowD = (size_t)p.D;
  const T* go = static_cast<const T*>(p.go) + (size_t)b * p.L * rowD + cc;
  const T* x = static_cast<const T*>(p.x) + (size_t)b * p.L * rowD + cc;
  T* dx = static_cast<T*>(p.dx) + (size_t)b * p.L * rowD + cc;
  const __nv_bfloat16* mean = p.mean + (size_t)b * p.L;
  const __nv_bfloat16* rstd = p.rstd + (size_t)b * p.L;
  const float invD = 1.0f / (float)p.D;

  float nw[4], cw[4][4];  // cw[e][k]
  ld4<T>(static_cast<const T*>(p.nw) + cc, nw);
#pragma unroll
  for (int e = 0; e < 4; ++e) ld4<T>(static_cast<const T*>(p.cw) + (size_t)(cc + e) * 4, cw[e]);

  auto load_go = [&](int t, float* f) {
    if (act && t < p.L) ld4<T>(go + (size_t)t * rowD, f);
    else f[0] = f[1] = f[2] = f[3] = 0.f;
  };
  auto xhat_nw = [&](int t, float* f) {  // xhat[t] * nw, zero for rows before the sequence
    if (act && t >= 0) {
      float v[4];
      ld4<T>(x + (size_t)t * rowD, v);
      const float m = __bfloat162float(mean[t]), r = __bfloat162float(rstd[t]);
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = (v[e] - m) * r * nw[e];
    } else {
      f[0] = f[1] = f[2] = f[3] = 0.f;
    }
  };
  // rings: G[rho & 3] = go row l0 + rho, X[rho & 3] = xhat * nw of row l0 + rho
  float G[4][4], X[4][4];
  load_go(l0, G[0]);
  load_go(l0 + 1, G[1]);
  load_go(l0 + 2, G[2]);
  xhat_nw(l0 - 3, X[1]);
  xhat_nw(l0 - 2, X[2]);
  xhat_nw(l0 - 1, X[3]);

  float a_nw[4] = {0.f, 0.f, 0.f, 0.f}, a_nb[4] = {0.f, 0.f, 0.f, 0.f}, a_cb[4] = {0.f, 0.f, 0.f, 0.f};
  float a_cw[4][4] = {};  // [k][e]
  int half = 0;
  for (int r4 = 0; r4 < l1 - l0; r4 += 4) {
    float xh[4][4], dxh[4][4], s1[4], s2[4], rs[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = l0 + r4 + u;
      s1[u] = s2[u] = 0.f;
      rs[u] = 0.f;
      if (t < l1) {
        load_go(t + 3, G[(u + 3) & 3]);
        float v[4];
        const float m = __bfloat162float(mean[t]), r = __bfloat162float(rstd[t]);
        rs[u] = r;
        if (act) ld4<T>(x + (size_t)t * rowD, v);
        else v[0] = v[1] = v[2] = v[3] = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float g0 = G[u][e];
          const float dn = g0 * cw[e][3] + G[(u + 1) & 3][e] * cw[e][2] + G[(u + 2) & 3][e] * cw[e][1] +
                           G[(u + 3) & 3][e] * cw[e][0];
          const float xhat = act ? (v[e] - m) * r : 0.f;
          const float xw = xhat * nw[e];
          xh[u][e] = xhat;
          dxh[u][e] = dn * nw[e];
          s1[u] += dxh[u][e];
          s2[u] += dxh[u][e] * xhat;
          a_nw[e] += dn * xhat;
          a_nb[e] += dn;
          a_cb[e] += g0;
          a_cw[3][e] += g0 * xw;
          a_cw[2][e] += g0 * X[(u + 3) & 3][e];
          a_cw[1][e] += g0 * X[(u + 2) & 3][e];
          a_cw[0][e] += g0 * X[(u + 1) & 3][e];
          X[u][e] = xw;
        }
      }
    }
    // the group's row sums over the CTA
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float a = warp_sum(s1[u]), c = warp_sum(s2[u]);
      if (lane == 0) {
        red[half][u][0][warp] = a;
        red[half][u][1][warp] = c;
      }
    }
    __syncthreads();
    // every warp reduces the warps' partials itself: one shared load per lane, then shuffles
    float S1v[4], S2v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      S1v[u] = warp_sum(lane < nwarps ? red[half][u][0][lane] : 0.f) * invD;
      S2v[u] = warp_sum(lane < nwarps ? red[half][u][1][lane] : 0.f) * invD;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = l0 + r4 + u;
      if (t >= l1 || !act) continue;
      const float S1 = S1v[u], S2 = S2v[u];
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = rs[u] * (dxh[u][e] - S1 - xh[u][e] * S2);
      st4<T>(dx + (size_t)t * rowD, o);
    }
    half ^= 1;
  }
  if (act) {
    float* part = p.part + (size_t)seg * 7 * rowD + c0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      part[e] = a_nw[e];
      part[rowD + e] = a_nb[e];
      part[2 * rowD + e] = a_cb[e];
#pragma unroll
      for (int k = 0; k < 4; ++k) part[(3 + k) * rowD + e] = a_cw[k][e];
    }
  }
}

// The same computation with the rows staged through shared memory: tile k of a CTA holds the
// x rows of its steps [l0 + k TR, +TR) and the grad rows three ahead, brought in by bulk TMA
// copies (rows are contiguous) into a ring of NST stages; a stage is refilled after the CTA
// barrier of the first 4-row group of the next tile.  Rows of a multiple of 16 bytes.
// The group's eight row sums (sum dn nw and sum dn nw xhat of 4 rows) reduce over the warp in
// one xor butterfly, over the warps through shared memory (one barrier per group); lane i of
// every warp fetches row i's mean / rstd once per tile (the rows take them by shuffle), and
// the arithmetic runs on packed fp32 pairs.

// Sum each of v[0..7] over the warp: lanes 4i..4i+3 end with the sum of value i (each xor
// level keeps half of the values and sends the other half to the partner).
__device__ __forceinline__ float warp_sum8(float* v, int lane) {
#pragma unroll
  for (int lvl = 0; lvl < 3; ++lvl) {
    const int half = 4 >> lvl;
    const bool up = (lane >> (4 - lvl)) & 1;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float keep = up ? v[half + i] : v[i];
      const float send = up ? v[i] : v[half + i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16 >> lvl);
    }
  }
  const float s = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 2);
  return s + __shfl_xor_sync(0xffffffffu, s, 1);
}

// four channels at a 32-bit shared address / in global memory <-> two fp32 pairs
template <typename T>
__device__ __forceinline__ void lds4(uint32_t a, uint64_t* f) {
  if constexpr (sizeof(T) == 4) {
    uint32_t x, y, z, w;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(x), "=r"(y), "=r"(z), "=r"(w) : "r"(a) : "memory");
    f[0] = f2_make(__uint_as_float(x), __uint_as_float(y));
    f[1] = f2_make(__uint_as_float(z), __uint_as_float(w));
  } else {
    uint32_t x, y;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(x), "=r"(y) : "r"(a) : "memory");
    f[0] = bf2_to_f2(x);
    f[1] = bf2_to_f2(y);
  }
}
template <typename T>
__device__ __forceinline__ void ldg4(const T* p, uint64_t* f) {
  float v[4];
  ld4<T>(p, v);
  f[0] = f2_make(v[0], v[1]);
  f[1] = f2_make(v[2], v[3]);
}
template <typename T>
__device__ __forceinline__ void stg4_if(T* p, const uint64_t* f, bool pred) {
  if constexpr (sizeof(T) == 4) {
    float a, b, c, d;
    f2_split(f[0], a, b);
    f2_split(f[1], c, d);
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t@q st.global.v4.f32 [%0], {%1,%2,%3,%4};\n\t}"
                 :: "l"(p), "f"(a), "f"(b), "f"(c), "f"(d), "r"((int)pred) : "memory");
  } else {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t@q st.global.v2.u32 [%0], {%1,%2};\n\t}"
                 :: "l"(p), "r"(f2_to_bf2(f[0])), "r"(f2_to_bf2(f[1])), "r"((int)pred) : "memory");
  }
}

template <typename T, int NST, int TR>
__global__ void __launch_bounds__(512) ln_conv_bwd_staged_kernel(LnConvBwdParams p) {
  static_assert(TR % 4 == 0 && TR <= 32, "tiles of whole 4-row groups, one row per lane");
  __shared__ __align__(16) float red[2][8][16];  // [half][value: 4 x sum dn nw, 4 x sum dn nw xhat][warp]
  extern __shared__ uint8_t smem_raw[];
  // 128-byte aligned by shared-space offset (pointer arithmetic on the array keeps accesses ld/st.shared)
  uint8_t* ring = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int seg = blockIdx.x;
  const int b = seg / p.segs_per_b;
  const int l0 = (seg - b * p.segs_per_b) * p.seg_len;
  const int l1 = min(l0 + p.seg_len, p.L);
  const int c0 = tid * 4;
  const bool act = c0 < p.D;
  const int cc = act ? c0 : p.D - 4;  // a thread past the row reads the last channels, stores nothing
  const size_t rowD = (size_t)p.D;
  const uint32_t row_bytes = (uint32_t)(p.D * sizeof(T));
  const uint32_t tile_bytes = (uint32_t)TR * row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + 2 * (size_t)NST * tile_bytes);  // [NST]
  const uint32_t ring_a = smem_u32(ring);
  const T* gob = static_cast<const T*>(p.go) + (size_t)b * p.L * rowD;
  const T* xb = static_cast<const T*>(p.x) + (size_t)b * p.L * rowD;
  T* dx = static_cast<T*>(p.dx) + (size_t)b * p.L * rowD + cc;
  const __nv_bfloat16* mean = p.mean + (size_t)b * p.L;
  const __nv_bfloat16* rstd = p.rstd + (size_t)b * p.L;
  const float invD = 1.0f / (float)p.D;
  const int ntiles = (l1 - l0 + TR - 1) / TR;

  if (tid == 0) {
    for (int i = 0; i < NST; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // tiles issued (thread 0)
  auto issue = [&](int k) {  // tile k: x rows t0.., grad rows t0+3.. (clipped to the sequence)
    const int st = k % NST;
    const int t0 = l0 + k * TR;
    const int nx = min(TR, l1 - t0);
    const int ng = max(0, min(TR, p.L - (t0 + 3)));
    uint8_t* sx = ring + (size_t)st * 2 * tile_bytes;
    mbar_expect_tx(&bars[st], (uint32_t)(nx + ng) * row_bytes);
    bulk_g2s(sx, xb + (size_t)t0 * rowD, (uint32_t)nx * row_bytes, &bars[st]);
    if (ng > 0) bulk_g2s(sx + tile_bytes, gob + (size_t)(t0 + 3) * rowD, (uint32_t)ng * row_bytes, &bars[st]);
    issued = k + 1;
  };
  if (tid == 0)
    for (int k = 0; k < NST && k < ntiles; ++k) issue(k);  // stage of tile k - 1 refilled at tile k

  // parameters as fp32 pairs: nw, and the taps c0..c3 of the channels (cw[e][k] of channel e)
  uint64_t nw2[2], c_0[2], c_1[2], c_2[2], c_3[2];
  {
    float nw[4], cw[4][4];
    ld4<T>(static_cast<const T*>(p.nw) + cc, nw);
#pragma unroll
    for (int e = 0; e < 4; ++e) ld4<T>(static_cast<const T*>(p.cw) + (size_t)(cc + e) * 4, cw[e]);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      nw2[j] = f2_make(nw[2 * j], nw[2 * j + 1]);
      c_0[j] = f2_make(cw[2 * j][0], cw[2 * j + 1][0]);
      c_1[j] = f2_make(cw[2 * j][1], cw[2 * j + 1][1]);
      c_2[j] = f2_make(cw[2 * j][2], cw[2 * j + 1][2]);
      c_3[j] = f2_make(cw[2 * j][3], cw[2 * j + 1][3]);
    }
  }
  // rings: G[rho & 3] = go row l0 + rho, X[rho & 3] = xhat * nw of row l0 + rho (rows before
  // the sequence: zero)
  uint64_t G[4][2], X[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) G[i][0] = G[i][1] = X[i][0] = X[i][1] = 0ull;
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    if (l0 + r < p.L) ldg4<T>(gob + (size_t)(l0 + r) * rowD + cc, G[r]);
    const int t = l0 - 3 + r;
    if (t >= 0) {
      uint64_t v[2];
      ldg4<T>(xb + (size_t)t * rowD + cc, v);
      const float m = __bfloat162float(mean[t]), rr = __bfloat162float(rstd[t]);
      const uint64_t r2 = f2_make(rr, rr), mr2 = f2_make(-m * rr, -m * rr);
#pragma unroll
      for (int j = 0; j < 2; ++j) X[r + 1][j] = f2_mul(f2_fma(v[j], r2, mr2), nw2[j]);
    }
  }

  uint64_t a_nw[2] = {0ull, 0ull}, a_nb[2] = {0ull, 0ull}, a_cb[2] = {0ull, 0ull};
  uint64_t a_cw[4][2] = {};  // [k][pair]
  int half = 0;
  bool ok = true;
  int k = 0;
  for (; k < ntiles && ok; ++k) {
    const int st = k % NST;
    const int t0 = l0 + k * TR;
    const int nrows = min(TR, l1 - t0);
    // row statistics of the tile: lane i holds row i's (TR <= 32)
    float mt = 0.f, rt = 0.f;
    if (lane < nrows) {
      mt = __bfloat162float(mean[t0 + lane]);
      rt = __bfloat162float(rstd[t0 + lane]);
    }
    // a timed-out wait ends the loop for every warp together at the group barrier below
    const bool got = mbar_wait_warp(&bars[st], (uint32_t)((k / NST) & 1), 34);
    const uint32_t sx = ring_a + (uint32_t)st * 2 * tile_bytes + (uint32_t)cc * sizeof(T);
    const uint32_t sg = sx + tile_bytes;
#pragma unroll
    for (int rk = 0; rk < TR; rk += 4) {  // the tile's groups, unrolled (TR is a compile-time constant)
      if (rk >= nrows) break;
      const int tg = t0 + rk;  // first row of the group
      uint64_t dxh[4][2];
      float v[8];
      // phase 1: dn, xhat, the row sums' partials, the parameter gradients
      auto row = [&](auto full, int u) {
        constexpr bool FULL = decltype(full)::value;
        const int t = tg + u, r = rk + u;
        const float m = __shfl_sync(0xffffffffu, mt, r & 31), rr = __shfl_sync(0xffffffffu, rt, r & 31);
        v[u] = v[4 + u] = 0.f;
        if (!FULL && t >= l1) return;
        if (FULL || t + 3 < p.L) lds4<T>(sg + (uint32_t)r * row_bytes, G[(u + 3) & 3]);
        else G[(u + 3) & 3][0] = G[(u + 3) & 3][1] = 0ull;
        uint64_t xv[2];
        lds4<T>(sx + (uint32_t)r * row_bytes, xv);
        const uint64_t r2 = f2_make(rr, rr), mr2 = f2_make(-m * rr, -m * rr);
        uint64_t s1 = 0ull, s2 = 0ull;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint64_t g0 = G[u][j];
          const uint64_t dn = f2_fma(G[(u + 3) & 3][j], c_0[j],
                                     f2_fma(G[(u + 2) & 3][j], c_1[j], f2_fma(G[(u + 1) & 3][j], c_2[j], f2_mul(g0, c_3[j]))));
          const uint64_t xhat = f2_fma(xv[j], r2, mr2);  // (x - mean) rstd
          const uint64_t xw = f2_mul(xhat, nw2[j]);
          const uint64_t d = f2_mul(dn, nw2[j]);
          dxh[u][j] = d;
          s1 = j ? f2_add(s1, d) : d;
          s2 = j ? f2_fma(d, xhat, s2) : f2_mul(d, xhat);
          a_nw[j] = f2_fma(dn, xhat, a_nw[j]);
          a_nb[j] = f2_add(a_nb[j], dn);
          a_cb[j] = f2_add(a_cb[j], g0);
          a_cw[3][j] = f2_fma(g0, xw, a_cw[3][j]);
          a_cw[2][j] = f2_fma(g0, X[(u + 3) & 3][j], a_cw[2][j]);
          a_cw[1][j] = f2_fma(g0, X[(u + 2) & 3][j], a_cw[1][j]);
          a_cw[0][j] = f2_fma(g0, X[(u + 1) & 3][j], a_cw[0][j]);
          X[u][j] = xw;
        }
        float lo, hi;
        f2_split(s1, lo, hi);
        v[u] = lo + hi;
        f2_split(s2, lo, hi);
        v[4 + u] = lo + hi;
      };
      const bool full = tg + 4 <= l1 && tg + 7 < p.L;
      if (full) {
        row(std::true_type{}, 0); row(std::true_type{}, 1); row(std::true_type{}, 2); row(std::true_type{}, 3);
      } else {
        row(std::false_type{}, 0); row(std::false_type{}, 1); row(std::false_type{}, 2); row(std::false_type{}, 3);
      }
      if (!act) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
      const float s = warp_sum8(v, lane);
      if ((lane & 3) == 0) red[half][lane >> 2][warp] = s;
      if (!__syncthreads_and(got)) { ok = false; break; }
      // every thread has finished tile k - 1 (its last group's phase 2 came before the barrier
      // above): refill that stage
      if (tid == 0 && rk == 0 && k >= 1 && k - 1 + NST < ntiles) {
        fence_proxy_async_smem();
        issue(k - 1 + NST);
      }
      // phase 2: every warp finishes the sums itself (lane i < 8: value i over the warps);
      // xhat is recomputed from the staged row
      // lane l adds value (l & 7) of warps 4 (l >> 3) .. +3; two xor levels join the four
      // quarters, so lanes 0..7 (and their copies) hold the eight sums
      float S = 0.f;
      {
        const int v = lane & 7, w0 = (lane >> 3) * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) S += (w0 + k < nwarps) ? red[half][v][w0 + k] : 0.f;
        S += __shfl_xor_sync(0xffffffffu, S, 8);
        S += __shfl_xor_sync(0xffffffffu, S, 16);
        S *= invD;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float S1 = __shfl_sync(0xffffffffu, S, u), S2 = __shfl_sync(0xffffffffu, S, 4 + u);
        const float m = __shfl_sync(0xffffffffu, mt, (rk + u) & 31), rr = __shfl_sync(0xffffffffu, rt, (rk + u) & 31);
        const int t = tg + u;
        if (t < l1) {
          const uint64_t r2 = f2_make(rr, rr), mr2 = f2_make(-m * rr, -m * rr);
          const uint64_t S1_2 = f2_make(S1, S1), mS2_2 = f2_make(-S2, -S2);
          uint64_t xv[2], o[2];
          lds4<T>(sx + (uint32_t)(rk + u) * row_bytes, xv);
#pragma unroll
          for (int j = 0; j < 2; ++j)
            o[j] = f2_mul(r2, f2_fma(f2_fma(xv[j], r2, mr2), mS2_2, f2_sub(dxh[u][j], S1_2)));
          stg4_if<T>(dx + (size_t)t * rowD, o, act);
        }
      }
      half ^= 1;
    }
    if (!ok) break;  // keep k at the tile whose copy timed out (waited for below)
  }
  if (act) {
    float* part = p.part + (size_t)seg * 7 * rowD + c0;
    auto put = [&](int row, const uint64_t* f) {
      float a, b2, c, d;
      f2_split(f[0], a, b2);
      f2_split(f[1], c, d);
      *reinterpret_cast<float4*>(part + (size_t)row * rowD) = make_float4(a, b2, c, d);
    };
    put(0, a_nw);
    put(1, a_nb);
    put(2, a_cb);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) put(3 + kk, a_cw[kk]);
  }
  // after a timed-out wait: let this CTA's own copies land (bounded) before exit
  if (!ok && tid == 0) {
    for (int j = k; j < issued; ++j) mbar_wait(&bars[j % NST], (uint32_t)((j / NST) & 1), 35);
  }
}

// sums the per-CTA partials [nseg][7][D] in CTA order and casts to T:
// dnw [D], dnb [D], dcb [D], dcw [D][4]
template <typename T>
__global__ void ln_conv_bwd_reduce_kernel(const float* part, int nseg, int D, T* dnw, T* dnb, T* dcw, T* dcb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (row of 7, channel)
  if (i >= 7 * D) return;
  const int k = i / D, d = i - k * D;
  float s = 0.f;
  // 16 loads in flight per thread (few threads: 7 D of them); the adds stay in CTA order
#pragma unroll 16
  for (int c = 0; c < nseg; ++c) s += part[(size_t)c * 7 * D + i];
  const T v = from_f<T>(s);
  if (k == 0) dnw[d] = v;
  else if (k == 1) dnb[d] = v;
  else if (k == 2) dcb[d] = v;
  else dcw[(size_t)d * 4 + (k - 3)] = v;
}

constexpr int kBwdMaxD = 2048;  // 512 threads x 4 channels

// one wave: a 512-thread CTA (D = 2048) per SM, more CTAs per SM for narrower rows
static void bwd_plan(int64_t B, int64_t L, int64_t D, int* seg_len, int* segs_per_b) {
  const int64_t threads = std::max<int64_t>(32, (D / 4 + 31) / 32 * 32);
  const int64_t target = (int64_t)num_sms() * std::max<int64_t>(1, std::min<int64_t>(4, 512 / threads));
  // segments per batch row rounded down: B * spb stays within one wave (rounding up gave
  // B = 8 on 148 SMs 152 CTAs, whose last 4 ran as a second wave of the whole CTA time)
  int64_t spb = std::max<int64_t>(1, target / B);
  int64_t len = (L + spb - 1) / spb;
  len = (len + 3) / 4 * 4;
  if (len < 16) len = 16;
  *seg_len = (int)len;
  *segs_per_b = (int)((L + len - 1) / len);
}

}  // namespace hdc

using namespace hdc;

extern "C" size_t hdc_ln_conv_bwd_workspace_bytes(int64_t B, int64_t L, int64_t D) {
  if (B < 1 || L < 1 || D < 1) return 0;
  int len, spb;
  bwd_plan(B, L, D, &len, &spb);
  return (size_t)B * spb * 7 * D * sizeof(float);
}

extern "C" int hdc_ln_conv_bwd(int dtype, const void* grad_out, const void* x, const void* mean, const void* rstd,
                               const void* norm_w, const void* conv_w, void* dx, void* dnorm_w, void* dnorm_b,
                               void* dconv_w, void* dconv_b, void* workspace, size_t workspace_bytes, int64_t B,
                               int64_t L, int64_t D, hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "ln_conv_bwd: dtype %d", dtype);
  if (!grad_out || !x || !mean || !rstd || !norm_w || !conv_w || !dx || !dnorm_w || !dnorm_b || !dconv_w ||
      !dconv_b || !workspace)
    return fail(HDC_E_NULL, "ln_conv_bwd: null pointer");
  if (B < 1 || L < 1 || D < 4 || D % 4 != 0 || D > kBwdMaxD || B * L > (int64_t)INT32_MAX)
    return fail(HDC_E_SHAPE, "ln_conv_bwd: B=%lld L=%lld D=%lld (D a multiple of 4, <= %d)", (long long)B,
                (long long)L, (long long)D, kBwdMaxD);
  const size_t need = hdc_ln_conv_bwd_workspace_bytes(B, L, D);
  if (workspace_bytes < need) return fail(HDC_E_WORKSPACE, "ln_conv_bwd: workspace %zu < %zu", workspace_bytes, need);
  if (!aligned16(grad_out) || !aligned16(x) || !aligned16(dx) || !aligned16(norm_w) || !aligned16(conv_w) ||
      !aligned16(workspace))
    return fail(HDC_E_ALIGN, "ln_conv_bwd: pointers must be 16-byte aligned");
  LnConvBwdParams p{};
  p.go = grad_out; p.x = x; p.mean = static_cast<const __nv_bfloat16*>(mean);
  p.rstd = static_cast<const __nv_bfloat16*>(rstd); p.nw = norm_w; p.cw = conv_w; p.dx = dx;
  p.part = static_cast<float*>(workspace); p.L = (int)L; p.D = (int)D;
  bwd_plan(B, L, D, &p.seg_len, &p.segs_per_b);
  const int nseg = (int)(B * p.segs_per_b);
  int threads = ((int)(D / 4) + 31) / 32 * 32;
  if (threads < 64) threads = 64;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const int rgrid = (int)((7 * D + 255) / 256);
  const size_t es = dtype == HDC_F32 ? 4 : 2;
  const size_t row_bytes = (size_t)D * es;
  const bool staged = row_bytes % 16 == 0;
  // 8-row tiles and 3 stages where they fit, else 4-row tiles, else 2 stages
  int TR = 8, nst = 3;
  auto smem_of = [&](int tr, int ns) { return 128 + 2 * (size_t)ns * tr * row_bytes + ns * 8 + 16; };
  if (smem_of(TR, nst) > 200 * 1024) TR = 4;
  if (smem_of(TR, nst) > 200 * 1024) nst = 2;
  const size_t smem = smem_of(TR, nst);
  auto launch_main = [&](auto tag) -> int {
    using T = decltype(tag);
    auto go = [&](auto kernel) {
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      kernel<<<nseg, threads, smem, s>>>(p);
    };
    if (!staged) ln_conv_bwd_kernel<T><<<nseg, threads, 0, s>>>(p);
    else if (nst == 3 && TR == 8) go(ln_conv_bwd_staged_kernel<T, 3, 8>);
    else if (nst == 3) go(ln_conv_bwd_staged_kernel<T, 3, 4>);
    else go(ln_conv_bwd_staged_kernel<T, 2, 4>);
    return launch_status("ln_conv_bwd_kernel");
  };
  if (dtype == HDC_F32) {
    if (int e = launch_main(float{})) return e;
    ln_conv_bwd_reduce_kernel<float><<<rgrid, 256, 0, s>>>(p.part, nseg, (int)D, static_cast<float*>(dnorm_w),
                                                           static_cast<float*>(dnorm_b), static_cast<float*>(dconv_w),
                                                           static_cast<float*>(dconv_b));
  } else {
    if (int e = launch_main(__nv_bfloat16{})) return e;
    ln_conv_bwd_reduce_kernel<__nv_bfloat16><<<rgrid, 256, 0, s>>>(
        p.part, nseg, (int)D, static_cast<__nv_bfloat16*>(dnorm_w), static_cast<__nv_bfloat16*>(dnorm_b),
        static_cast<__nv_bfloat16*>(dconv_w), static_cast<__nv_bfloat16*>(dconv_b));
  }
  return launch_status("ln_conv_bwd_reduce_kernel");
}
