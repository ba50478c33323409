// Fused LayerNorm + causal depthwise conv1d (width 4) (+ optional SiLU), sm_100a.
//
// Same math as the reference _fused_norm_conv_fwd_kernel (hdcmamba/model.py:22-72):
//   n[t]   = (x[t] - mean_t) * rstd_t * norm_w + norm_b          (fp32, two-pass variance)
//   out[t] = n[t-3]*cw0 + n[t-2]*cw1 + n[t-1]*cw2 + n[t]*cw3 + cb
// with rows t < 0 equal to zeros (LayerNorm(0) = norm_b) or to a supplied halo.
//
// Layout and schedule (HBM-bound: every x byte read once, every out byte written once):
//   * a "group" of GP threads (whole warps) owns one contiguous L-segment of one batch
//     row; thread g of the group owns VPT 16-byte column vectors (channels
//     [VEC*(g + k*GP), +VEC)).  Each CTA holds S = blockDim/GP groups.
//   * the group walks its segment TILE rows at a time.  The next tile's 16-byte loads
//     are issued before the current tile is reduced, so loads stay in flight.
//   * per-row mean/variance: per-thread partials -> warp shuffles -> a per-group
//     named barrier (bar.sync 1+s, GP) -> partials of the group's warps summed.
//   * the three previous normalised rows live in registers (the conv window), so no
//     row is read twice except the 3 rows before each segment.
#include "common.cuh"

namespace hdc {

struct LnConvParams {
  const void* x; const void* nw; const void* nb; const void* cw; const void* cb;
  const void* halo; void* out; __nv_bfloat16* mean; __nv_bfloat16* rstd;
  int L, D, seg_len, segs_per_b, total_segs, group_threads;
  float eps; int act;
};

__device__ __forceinline__ void group_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <typename T, int VPT, int TILE>
__global__ void __launch_bounds__(256) ln_conv_kernel(LnConvParams p) {
  constexpr int VEC = Vec<T>::N;
  // reduction scratch: [2 buffers][S groups][8 warps][TILE]
  __shared__ float red[2][8][8][TILE];

  const int GP = p.group_threads;
  const int s = threadIdx.x / GP;
  const int g = threadIdx.x - s * GP;
  const int warp = g >> 5, lane = threadIdx.x & 31, nwarp = GP >> 5;
  const int seg = blockIdx.x * (blockDim.x / GP) + s;
  if (seg >= p.total_segs) return;  // the whole group leaves together
  const int b = seg / p.segs_per_b;
  const int l0 = (seg - b * p.segs_per_b) * p.seg_len;
  const int l1 = min(l0 + p.seg_len, p.L);
  const int G = p.D / VEC;
  const float invD = 1.0f / (float)p.D;

  const T* __restrict__ x = static_cast<const T*>(p.x) + (size_t)b * p.L * p.D;
  const T* __restrict__ halo = p.halo ? static_cast<const T*>(p.halo) + (size_t)b * 3 * p.D : nullptr;
  T* __restrict__ out = static_cast<T*>(p.out) + (size_t)b * p.L * p.D;

  // Parameters for this thread's channels, kept packed (16 bytes per vector).
  uint4 pnw[VPT], pnb[VPT], pcb[VPT], pcw[4][VPT];
  bool active[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = g + k * GP;
    active[k] = c < G;
    if (active[k]) {
      pnw[k] = ldg16(static_cast<const T*>(p.nw) + c * VEC);
      pnb[k] = ldg16(static_cast<const T*>(p.nb) + c * VEC);
      pcb[k] = ldg16(static_cast<const T*>(p.cb) + c * VEC);
      // conv_w is [D, 4]: de-interleave the 4 taps of VEC channels
      const T* cwp = static_cast<const T*>(p.cw) + (size_t)c * VEC * 4;
      float taps[4][VEC];
#pragma unroll
      for (int q = 0; q < VEC * 4 / Vec<T>::N; ++q) {
        float f[Vec<T>::N];
        unpack16<T>(ldg16(cwp + q * Vec<T>::N), f);
#pragma unroll
        for (int e = 0; e < Vec<T>::N; ++e) {
          const int flat = q * Vec<T>::N + e;
          taps[flat & 3][flat >> 2] = f[e];
        }
      }
#pragma unroll
      for (int tp = 0; tp < 4; ++tp) pcw[tp][k] = pack16<T>(taps[tp]);
    } else {
      pnw[k] = pnb[k] = pcb[k] = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int tp = 0; tp < 4; ++tp) pcw[tp][k] = make_uint4(0, 0, 0, 0);
    }
  }

  auto row_ptr = [&](int t) -> const T* {
    if (t >= 0) return x + (size_t)t * p.D;
    if (halo) return halo + (size_t)(3 + t) * p.D;
    return nullptr;  // zero row
  };
  auto load_tile = [&](uint4 (&buf)[TILE][VPT], int t0, int nvalid) {
#pragma unroll
    for (int r = 0; r < TILE; ++r) {
      const T* rp = (r < nvalid) ? row_ptr(t0 + r) : nullptr;
#pragma unroll
      for (int k = 0; k < VPT; ++k)
        buf[r][k] = (rp && active[k]) ? ldg16(rp + (g + k * GP) * VEC) : make_uint4(0, 0, 0, 0);
    }
  };
  // group-wide sum of TILE per-thread partials, result broadcast to all threads
  auto group_sum = [&](float (&v)[TILE], int bufi) {
#pragma unroll
    for (int r = 0; r < TILE; ++r) v[r] = warp_sum(v[r]);
    if (nwarp == 1) return;
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < TILE; ++r) red[bufi][s][warp][r] = v[r];
    }
    group_bar(1 + s, GP);
#pragma unroll
    for (int r = 0; r < TILE; ++r) {
      float acc = 0.f;
      for (int w = 0; w < nwarp; ++w) acc += red[bufi][s][w][r];
      v[r] = acc;
    }
  };
  // mean / rstd of a tile of rows held in `buf`
  auto tile_stats = [&](const uint4 (&buf)[TILE][VPT], float (&mean)[TILE], float (&rstd)[TILE]) {
    float f[VEC];
#pragma unroll
    for (int r = 0; r < TILE; ++r) {
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        unpack16<T>(buf[r][k], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) sum += f[e];
      }
      mean[r] = sum;
    }
    group_sum(mean, 0);
#pragma unroll
    for (int r = 0; r < TILE; ++r) mean[r] *= invD;
#pragma unroll
    for (int r = 0; r < TILE; ++r) {
      float sq = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!active[k]) continue;
        unpack16<T>(buf[r][k], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float d = f[e] - mean[r];
          sq += d * d;
        }
      }
      rstd[r] = sq;
    }
    group_sum(rstd, 1);
#pragma unroll
    for (int r = 0; r < TILE; ++r) rstd[r] = rsqrtf(rstd[r] * invD + p.eps);
  };

  // conv window: normalised rows t-3, t-2, t-1 (fp32)
  float w3[VPT][VEC], w2[VPT][VEC], w1[VPT][VEC];
  {
    uint4 hb[TILE][VPT];
    static_assert(TILE >= 3, "TILE must cover the 3-row halo");
    load_tile(hb, l0 - 3, 3);
    float hm[TILE], hr[TILE];
    tile_stats(hb, hm, hr);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      float f[VEC], nw[VEC], nb[VEC];
      unpack16<T>(pnw[k], nw);
      unpack16<T>(pnb[k], nb);
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        unpack16<T>(hb[r][k], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float n = (f[e] - hm[r]) * hr[r] * nw[e] + nb[e];
          if (r == 0) w3[k][e] = n; else if (r == 1) w2[k][e] = n; else w1[k][e] = n;
        }
      }
    }
  }

  uint4 cur[TILE][VPT], nxt[TILE][VPT];
  load_tile(cur, l0, min(TILE, l1 - l0));
  for (int t0 = l0; t0 < l1; t0 += TILE) {
    const int nv = min(TILE, l1 - t0);
    if (t0 + TILE < l1) load_tile(nxt, t0 + TILE, min(TILE, l1 - t0 - TILE));
    float mean[TILE], rstd[TILE];
    tile_stats(cur, mean, rstd);
    if (p.mean && g == 0) {
#pragma unroll
      for (int r = 0; r < TILE; ++r)
        if (r < nv) {
          p.mean[(size_t)b * p.L + t0 + r] = __float2bfloat16_rn(mean[r]);
          p.rstd[(size_t)b * p.L + t0 + r] = __float2bfloat16_rn(rstd[r]);
        }
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      float nw[VEC], nb[VEC], c0[VEC], c1[VEC], c2[VEC], c3[VEC], cb[VEC], f[VEC], o[VEC];
      unpack16<T>(pnw[k], nw); unpack16<T>(pnb[k], nb); unpack16<T>(pcb[k], cb);
      unpack16<T>(pcw[0][k], c0); unpack16<T>(pcw[1][k], c1);
      unpack16<T>(pcw[2][k], c2); unpack16<T>(pcw[3][k], c3);
#pragma unroll
      for (int r = 0; r < TILE; ++r) {
        if (r >= nv) break;
        unpack16<T>(cur[r][k], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float n0 = (f[e] - mean[r]) * rstd[r] * nw[e] + nb[e];
          float v = w3[k][e] * c0[e] + w2[k][e] * c1[e] + w1[k][e] * c2[e] + n0 * c3[e] + cb[e];
          if (p.act == HDC_ACT_SILU) v = v / (1.0f + expf(-v));
          o[e] = v;
          w3[k][e] = w2[k][e]; w2[k][e] = w1[k][e]; w1[k][e] = n0;
        }
        if (active[k]) stg16(out + (size_t)(t0 + r) * p.D + (g + k * GP) * VEC, pack16<T>(o));
      }
    }
#pragma unroll
    for (int r = 0; r < TILE; ++r)
#pragma unroll
      for (int k = 0; k < VPT; ++k) cur[r][k] = nxt[r][k];
  }
}

template <typename T, int VPT, int TILE>
static int launch_ln_conv(LnConvParams p, int64_t B, cudaStream_t stream) {
  const int G = p.D / Vec<T>::N;
  const int per = (G + VPT - 1) / VPT;
  const int GP = ((per + 31) / 32) * 32;
  const int S = GP >= 256 ? 1 : 256 / GP;
  const int threads = GP * S;
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ln_conv_kernel<T, VPT, TILE>, threads, 0);
  if (occ < 1) occ = 1;
  const int64_t target_groups = (int64_t)num_sms() * occ * S;
  int64_t segs_per_b = (target_groups + B - 1) / B;
  int64_t seg_len = (p.L + segs_per_b - 1) / segs_per_b;
  seg_len = ((seg_len + TILE - 1) / TILE) * TILE;
  if (seg_len < 4) seg_len = 4;
  segs_per_b = (p.L + seg_len - 1) / seg_len;
  p.seg_len = (int)seg_len;
  p.segs_per_b = (int)segs_per_b;
  p.total_segs = (int)(B * segs_per_b);
  p.group_threads = GP;
  const int grid = (p.total_segs + S - 1) / S;
  ln_conv_kernel<T, VPT, TILE><<<grid, threads, 0, stream>>>(p);
  return launch_status("ln_conv_kernel");
}

template <typename T>
static int ln_conv_dispatch(LnConvParams p, int64_t B, cudaStream_t stream) {
  const int G = p.D / Vec<T>::N;
  if (G <= 256) return launch_ln_conv<T, 1, 8>(p, B, stream);
  if (G <= 512) return launch_ln_conv<T, 2, 4>(p, B, stream);
  if (G <= 1024) return launch_ln_conv<T, 4, 4>(p, B, stream);
  return fail(HDC_E_SHAPE, "ln_conv: D=%d too large", p.D);
}

}  // namespace hdc

using namespace hdc;

extern "C" int hdc_ln_conv_fwd(int dtype, const void* x, const void* norm_w, const void* norm_b,
                               const void* conv_w, const void* conv_b, const void* halo, void* out,
                               void* mean, void* rstd, int64_t B, int64_t L, int64_t D, float eps,
                               int act, hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "ln_conv: dtype %d", dtype);
  if (!x || !norm_w || !norm_b || !conv_w || !conv_b || !out) return fail(HDC_E_NULL, "ln_conv: null pointer");
  if ((mean == nullptr) != (rstd == nullptr)) return fail(HDC_E_NULL, "ln_conv: mean and rstd go together");
  const int vec = dtype == HDC_F32 ? 4 : 8;
  if (B < 1 || L < 1 || D < vec || D % vec != 0 || D > 8192 || B * L > (int64_t)INT32_MAX)
    return fail(HDC_E_SHAPE, "ln_conv: B=%lld L=%lld D=%lld (D must be a multiple of %d, <= 8192)",
                (long long)B, (long long)L, (long long)D, vec);
  if (act != HDC_ACT_NONE && act != HDC_ACT_SILU) return fail(HDC_E_SHAPE, "ln_conv: act %d", act);
  if (!aligned16(x) || !aligned16(out) || !aligned16(norm_w) || !aligned16(norm_b) || !aligned16(conv_w) ||
      !aligned16(conv_b) || (halo && !aligned16(halo)))
    return fail(HDC_E_ALIGN, "ln_conv: pointers must be 16-byte aligned");
  if (x == out) return fail(HDC_E_SHAPE, "ln_conv: out must not alias x");
  LnConvParams p{};
  p.x = x; p.nw = norm_w; p.nb = norm_b; p.cw = conv_w; p.cb = conv_b; p.halo = halo; p.out = out;
  p.mean = static_cast<__nv_bfloat16*>(mean); p.rstd = static_cast<__nv_bfloat16*>(rstd);
  p.L = (int)L; p.D = (int)D; p.eps = eps; p.act = act;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  return dtype == HDC_F32 ? ln_conv_dispatch<float>(p, B, s) : ln_conv_dispatch<__nv_bfloat16>(p, B, s);
}
