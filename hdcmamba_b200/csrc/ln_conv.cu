// Fused LayerNorm + causal depthwise conv1d (width 4) (+ optional SiLU), sm_100a.
//
// Same math as the reference _fused_norm_conv_fwd_kernel (hdcmamba/model.py:22-72):
//   n[t]   = (x[t] - mean_t) * rstd_t * norm_w + norm_b          (fp32, two-pass variance)
//   out[t] = n[t-3]*cw0 + n[t-2]*cw1 + n[t-1]*cw2 + n[t]*cw3 + cb
// with rows t < 0 equal to zeros (LayerNorm(0) = norm_b) or to a supplied halo.
//
// Layout and schedule (HBM-bound; every x byte is read from DRAM once, every out byte
// written once):
//   * one CTA walks a contiguous L-segment of one batch row; thread g owns the 16-byte
//     channel vector g (and g + blockDim when D needs two vectors per thread).
//   * rows arrive through a ring of NST shared-memory stages filled by one-dimensional
//     bulk TMA copies (cp.async.bulk, mbarrier completion): a stage is TILE consecutive
//     rows, which are contiguous in memory.  The copy of tile k+NST is issued as soon
//     as tile k has been consumed.
//   * per-row mean / rstd: one warp per row reads the row from shared memory (the whole
//     row is in the stage), two-pass variance with warp shuffles only.  The statistics of
//     tile k+1 are computed in the same phase as the conv of tile k (one barrier per tile).
//   * the conv walks the tile's rows with the three previous normalised rows held in
//     registers, so each thread's window carries from tile to tile.
#include "tc.cuh"

namespace hdc {

struct LnConvParams {
  const void* x; const void* nw; const void* nb; const void* cw; const void* cb;
  const void* halo; void* out; __nv_bfloat16* mean; __nv_bfloat16* rstd;
  int L, D, seg_len, segs_per_b, total_segs, tile, nst;
  float eps; int act;
};


template <typename T, int VPT, bool SILU>
__global__ void __launch_bounds__(512) ln_conv_kernel(LnConvParams p) {
  constexpr int VEC = Vec<T>::N;
  extern __shared__ uint8_t smem_raw[];
  const int row_bytes = p.D * (int)sizeof(T);
  const int G = p.D / VEC;
  // smem: [nst][tile] rows | 3 pre rows | stats [nst][tile][2] + pre-row stats [3][2] |
  // mbarriers [nst + 1]
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* pre = ring + (size_t)p.nst * p.tile * row_bytes;
  float* stats = reinterpret_cast<float*>(pre + 3 * row_bytes);
  float* pstats = stats + 2 * p.nst * p.tile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(pstats + 6);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int seg = blockIdx.x;
  const int b = seg / p.segs_per_b;
  const int l0 = (seg - b * p.segs_per_b) * p.seg_len;
  const int l1 = min(l0 + p.seg_len, p.L);
  const int ntiles = (l1 - l0 + p.tile - 1) / p.tile;
  const T* __restrict__ x = static_cast<const T*>(p.x) + (size_t)b * p.L * p.D;
  T* __restrict__ out = static_cast<T*>(p.out) + (size_t)b * p.L * p.D;
  const float invD = 1.0f / (float)p.D;

  if (tid == 0) {
    for (int i = 0; i <= p.nst; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int k) {
    const int t0 = l0 + k * p.tile;
    const int nv = min(p.tile, l1 - t0);
    uint64_t* bar = &bars[k % p.nst];
    mbar_expect_tx(bar, (uint32_t)(nv * row_bytes));
    bulk_g2s(ring + (size_t)(k % p.nst) * p.tile * row_bytes, x + (size_t)t0 * p.D, (uint32_t)(nv * row_bytes), bar);
  };
  // the three rows before the segment: x rows, the halo, or zeros
  const bool pre_zero = (l0 == 0 && p.halo == nullptr);
  if (tid == 0) {
    for (int k = 0; k < p.nst && k < ntiles; ++k) issue(k);
    if (!pre_zero) {
      const T* src = l0 > 0 ? x + (size_t)(l0 - 3) * p.D : static_cast<const T*>(p.halo) + (size_t)b * 3 * p.D;
      mbar_expect_tx(&bars[p.nst], (uint32_t)(3 * row_bytes));
      bulk_g2s(pre, src, (uint32_t)(3 * row_bytes), &bars[p.nst]);
    }
  }
  if (pre_zero) {
    for (int i = tid; i < 3 * row_bytes / 16; i += blockDim.x) reinterpret_cast<uint4*>(pre)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();  // the zero rows are read by every warp below
  } else {
    mbar_wait(&bars[p.nst], 0, 31);
  }

  // per-row statistics of `nrows` rows at `rows`, one warp per row -> st[2*r], st[2*r+1]
  // (two passes over the row in shared memory: mean, then the centred sum of squares)
  auto row_stats = [&](const uint8_t* rows, int nrows, float* st) {
    for (int r = warp; r < nrows; r += nwarps) {
      const uint4* rp = reinterpret_cast<const uint4*>(rows + (size_t)r * row_bytes);
      float s = 0.f;
      for (int c = lane; c < G; c += 32) {
        float f[VEC];
        unpack16<T>(rp[c], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) s += f[e];
      }
      const float mean = warp_sum(s) * invD;
      float q = 0.f;
      for (int c = lane; c < G; c += 32) {
        float f[VEC];
        unpack16<T>(rp[c], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float d = f[e] - mean;
          q = fmaf(d, d, q);
        }
      }
      const float rstd = rsqrtf(warp_sum(q) * invD + p.eps);
      if (lane == 0) {
        st[2 * r] = mean;
        st[2 * r + 1] = rstd;
      }
    }
  };

  // parameters of this thread's channels
  float nw[VPT][VEC], nb[VPT][VEC], c0[VPT][VEC], c1[VPT][VEC], c2[VPT][VEC], c3[VPT][VEC], cb[VPT][VEC];
  bool active[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = tid + k * blockDim.x;
    active[k] = c < G;
    const int cc = active[k] ? c : 0;
    unpack16<T>(ldg16(static_cast<const T*>(p.nw) + cc * VEC), nw[k]);
    unpack16<T>(ldg16(static_cast<const T*>(p.nb) + cc * VEC), nb[k]);
    unpack16<T>(ldg16(static_cast<const T*>(p.cb) + cc * VEC), cb[k]);
    const T* cwp = static_cast<const T*>(p.cw) + (size_t)cc * VEC * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f[VEC];
      unpack16<T>(ldg16(cwp + q * VEC), f);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int flat = q * VEC + e, ch = flat >> 2, tap = flat & 3;
        if (tap == 0) c0[k][ch] = f[e];
        else if (tap == 1) c1[k][ch] = f[e];
        else if (tap == 2) c2[k][ch] = f[e];
        else c3[k][ch] = f[e];
      }
    }
  }

  // conv window: W[k][rho & 3] holds the normalised row rho (relative to the segment start,
  // rows -3..-1 from the preceding rows), so with tiles of a multiple of 4 rows and the row
  // loop unrolled by 4 every index is a compile-time constant (no register moves)
  float W[VPT][4][VEC];
  row_stats(pre, 3, pstats);
  bool ok = true;
  if (ntiles > 0) {  // statistics of tile 0 (those of tile k+1 are computed next to tile k's conv)
    ok = mbar_wait(&bars[0], 0, 32);
    if (ok) row_stats(ring, min(p.tile, l1 - l0), stats);
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = active[k] ? tid + k * blockDim.x : 0;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      float f[VEC];
      unpack16<T>(reinterpret_cast<const uint4*>(pre + (size_t)r * row_bytes)[c], f);
      // the same expression as the row loop, so a halo row normalises to the same bits
      const float rs = pstats[2 * r + 1], mrs = -pstats[2 * r] * rs;
#pragma unroll
      for (int e = 0; e < VEC; ++e) W[k][r + 1][e] = fmaf(fmaf(f[e], rs, mrs), nw[k][e], nb[k][e]);
    }
  }

  for (int k = 0; k < ntiles && ok; ++k) {
    const int st = k % p.nst;
    const int t0 = l0 + k * p.tile;
    const int nv = min(p.tile, l1 - t0);
    const uint8_t* tile = ring + (size_t)st * p.tile * row_bytes;
    const float* tstat = stats + 2 * st * p.tile;
    if (k + 1 < ntiles) {  // the next tile's row statistics, in the same phase as this conv
      const int st1 = (k + 1) % p.nst;
      if (!mbar_wait(&bars[st1], (uint32_t)(((k + 1) / p.nst) & 1), 32)) { ok = false; break; }
      row_stats(ring + (size_t)st1 * p.tile * row_bytes, min(p.tile, l1 - (t0 + p.tile)), stats + 2 * st1 * p.tile);
    }
    if (p.mean && tid < nv) {
      p.mean[(size_t)b * p.L + t0 + tid] = __float2bfloat16_rn(tstat[2 * tid]);
      p.rstd[(size_t)b * p.L + t0 + tid] = __float2bfloat16_rn(tstat[2 * tid + 1]);
    }
#pragma unroll
    for (int kk = 0; kk < VPT; ++kk) {
      if (!active[kk]) continue;
      const int c = tid + kk * blockDim.x;
      for (int r4 = 0; r4 < nv; r4 += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = r4 + u;
          if (r < nv) {
            float f[VEC], o[VEC];
            unpack16<T>(reinterpret_cast<const uint4*>(tile + (size_t)r * row_bytes)[c], f);
            const float rs = tstat[2 * r + 1], mrs = -tstat[2 * r] * rs;
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              const float n0 = fmaf(fmaf(f[e], rs, mrs), nw[kk][e], nb[kk][e]);  // (x - mean) rstd w + b
              float v = fmaf(W[kk][(u + 1) & 3][e], c0[kk][e],
                             fmaf(W[kk][(u + 2) & 3][e], c1[kk][e],
                                  fmaf(W[kk][(u + 3) & 3][e], c2[kk][e], fmaf(n0, c3[kk][e], cb[kk][e]))));
              if (SILU) v *= fast_sigmoid(v);
              o[e] = v;
              W[kk][u][e] = n0;
            }
            stg16(out + (size_t)(t0 + r) * p.D + c * VEC, pack16<T>(o));
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0 && k + p.nst < ntiles) {
      fence_proxy_async_smem();  // order this stage's generic reads before the async refill
      issue(k + p.nst);
    }
  }
  // after a timed-out wait: let this CTA's own copies in flight land (bounded) before exit
  if (!ok && tid == 0) {
    for (int k = 0; k < ntiles && k < p.nst; ++k) mbar_wait(&bars[k], 0, 33);
  }
}

template <typename T, int VPT, bool SILU>
static int launch_ln_conv(LnConvParams p, int64_t B, cudaStream_t stream) {
  const int G = p.D / Vec<T>::N;
  int threads = ((G + VPT - 1) / VPT + 31) / 32 * 32;
  if (threads < 128) threads = 128;
  const int row_bytes = p.D * (int)sizeof(T);
  // stages of 32 KB for rows of 4 KB and more (8 rows: one per warp for the statistics),
  // 16 KB otherwise (shorter segments keep more CTAs busy at narrow rows); a multiple of 4
  // rows (the conv window unroll)
  int tile = ((row_bytes >= 4096 ? 32768 : 16384) / row_bytes) & ~3;
  tile = tile < 4 ? 4 : (tile > 16 ? 16 : tile);
  int nst = 3;
  auto smem_of = [&](int t, int s) {
    return (size_t)128 + (size_t)s * t * row_bytes + 3 * (size_t)row_bytes + (2 * s * t + 6) * 4 + (s + 1) * 8 + 16;
  };
  while (smem_of(tile, nst) > 110 * 1024 && nst > 2) --nst;
  while (smem_of(tile, nst) > 200 * 1024 && tile > 4) tile -= 4;
  const size_t smem = smem_of(tile, nst);
  cudaFuncSetAttribute(ln_conv_kernel<T, VPT, SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ln_conv_kernel<T, VPT, SILU>, threads, smem);
  if (occ < 1) occ = 1;
  const int64_t target = (int64_t)num_sms() * occ;
  int64_t segs_per_b = (target + B - 1) / B;
  int64_t seg_len = (p.L + segs_per_b - 1) / segs_per_b;
  seg_len = ((seg_len + tile - 1) / tile) * tile;
  if (seg_len < 8) seg_len = 8;
  segs_per_b = (p.L + seg_len - 1) / seg_len;
  p.seg_len = (int)seg_len;
  p.segs_per_b = (int)segs_per_b;
  p.total_segs = (int)(B * segs_per_b);
  p.tile = tile;
  p.nst = nst;
  ln_conv_kernel<T, VPT, SILU><<<p.total_segs, threads, smem, stream>>>(p);
  return launch_status("ln_conv_kernel");
}

template <typename T>
static int ln_conv_dispatch(LnConvParams p, int64_t B, cudaStream_t stream) {
  const int G = p.D / Vec<T>::N;
  if (G <= 512)
    return p.act == HDC_ACT_SILU ? launch_ln_conv<T, 1, true>(p, B, stream) : launch_ln_conv<T, 1, false>(p, B, stream);
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
  if (B < 1 || L < 1 || D < vec || D % vec != 0 || D > 512 * vec || B * L > (int64_t)INT32_MAX)
    return fail(HDC_E_SHAPE, "ln_conv: B=%lld L=%lld D=%lld (D must be a multiple of %d, <= %d)",
                (long long)B, (long long)L, (long long)D, vec, 512 * vec);
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
