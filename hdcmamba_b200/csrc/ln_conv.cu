// Fused LayerNorm + causal depthwise conv1d (width 4) (+ optional SiLU), sm_100a.
//
// Same math as the reference _fused_norm_conv_fwd_kernel (hdcmamba/model.py:22-72):
//   n[t]   = (x[t] - mean_t) * rstd_t * norm_w + norm_b          (fp32)
//   out[t] = n[t-3]*cw0 + n[t-2]*cw1 + n[t-1]*cw2 + n[t]*cw3 + cb
// with rows t < 0 equal to zeros (LayerNorm(0) = norm_b) or to a supplied halo.  The kernel
// carries the pre-affine rows z[t] = (x[t] - mean_t) * rstd_t through the conv window and
// applies the affine once: out = norm_w * sum_k cw_k z[t-3+k] + (norm_b * sum_k cw_k + cb)
// (the same value in fp32 up to reassociation; a zero row has z = 0).
//
// Layout and schedule (HBM-bound; every x byte is read from DRAM once, every out byte
// written once):
//   * one CTA walks a contiguous L-segment of one batch row with one thread per 16-byte
//     channel vector (blockDim = D / vector, rounded up to a warp), so thread c owns the
//     same channels in every row and keeps their conv window in registers.
//   * rows arrive through a ring of NST shared-memory stages of 8 rows, each filled by one
//     one-dimensional bulk copy (cp.async.bulk, mbarrier completion): the rows of one batch
//     are contiguous.  Tile k + NST - 1 is issued as soon as tile k - 1 has been consumed.
//   * row statistics come from the same threads: each sums its 8 channels of the 8 rows,
//     shifted by the row's first element (sum d, sum d^2 with d = x - x[row, 0]; one pass),
//     the 16 sums reduce over the warp in one xor butterfly, over the warps through shared
//     memory (one barrier per tile), and every warp finalises mean / rstd for itself.  The
//     summation order of a row does not depend on where the row sits in a tile, so a
//     segment that starts with a halo reproduces the unsplit run bit for bit.
//   * the arithmetic runs on packed fp32 pairs (add / mul / fma .f32x2).
#include <type_traits>

#include "flag.cuh"

namespace hdc {

struct LnConvParams {
  const void* x; const void* nw; const void* nb; const void* cw; const void* cb;
  const void* halo; void* out; __nv_bfloat16* mean; __nv_bfloat16* rstd;
  // sequence parallelism: the halo arrives from another GPU; the CTAs that read it wait
  // (bounded) until *halo_flag reaches *halo_gen (nullptr: no wait)
  const uint32_t* halo_flag; const uint32_t* halo_gen;
  int L, D, seg_len, segs_per_b, total_segs, nst;
  float eps; int act;
};

constexpr int LNC_ROWS = 8;  // rows per stage (a multiple of 4: the conv window rotates mod 4)

// 16-byte vector of T <-> fp32 pairs (NP = elements / 2)
template <typename T>
__device__ __forceinline__ void vec_to_f2(const uint4& u, uint64_t* p) {
  if constexpr (sizeof(T) == 4) {
    p[0] = f2_make(__uint_as_float(u.x), __uint_as_float(u.y));
    p[1] = f2_make(__uint_as_float(u.z), __uint_as_float(u.w));
  } else {
    p[0] = bf2_to_f2(u.x); p[1] = bf2_to_f2(u.y); p[2] = bf2_to_f2(u.z); p[3] = bf2_to_f2(u.w);
  }
}
template <typename T>
__device__ __forceinline__ uint4 f2_to_vec(const uint64_t* p) {
  if constexpr (sizeof(T) == 4) {
    float a, b, c, d;
    f2_split(p[0], a, b);
    f2_split(p[1], c, d);
    return make_uint4(__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d));
  } else {
    return make_uint4(f2_to_bf2(p[0]), f2_to_bf2(p[1]), f2_to_bf2(p[2]), f2_to_bf2(p[3]));
  }
}

// 16-byte / one-element shared-memory loads at 32-bit shared addresses
__device__ __forceinline__ uint4 lds16(uint32_t a) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a) : "memory");
  return r;
}
template <typename T>
__device__ __forceinline__ float lds_elem(uint32_t a) {
  if constexpr (sizeof(T) == 4) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
  } else {
    uint16_t h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a) : "memory");
    return __uint_as_float((uint32_t)h << 16);
  }
}
// 16-byte global store when `pred` (one predicated instruction, no branch)
__device__ __forceinline__ void stg16_if(void* p, const uint4& v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
               "@q st.global.v4.u32 [%0], {%1,%2,%3,%4};\n\t}"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"((int)pred) : "memory");
}

// This thread's shifted sums over the rows of a stage (vector at `va` in row 0, rows
// `row_bytes` apart; all R rows when FULL, else the first `nv`):
// v[r] = sum (x - K_r), v[8 + r] = sum (x - K_r)^2, K_r = element 0 of row r (at `ka` + r *
// row_bytes); zeros for the other rows.
template <typename T, bool FULL>
__device__ __forceinline__ void row_partials(uint32_t va, uint32_t ka, int row_bytes, int nv, float* v) {
  constexpr int NP = Vec<T>::N / 2;
#pragma unroll
  for (int r = 0; r < LNC_ROWS; ++r) {
    v[r] = 0.f;
    v[LNC_ROWS + r] = 0.f;
    if (FULL || r < nv) {
      const float K = lds_elem<T>(ka + r * row_bytes);
      const uint64_t K2 = f2_make(K, K);
      uint64_t xp[NP];
      vec_to_f2<T>(lds16(va + r * row_bytes), xp);
      uint64_t d = f2_sub(xp[0], K2);
      uint64_t s1 = d, s2 = f2_mul(d, d);
#pragma unroll
      for (int j = 1; j < NP; ++j) {
        d = f2_sub(xp[j], K2);
        s1 = f2_add(s1, d);
        s2 = f2_fma(d, d, s2);
      }
      float x0, x1;
      f2_split(s1, x0, x1);
      v[r] = x0 + x1;
      f2_split(s2, x0, x1);
      v[LNC_ROWS + r] = x0 + x1;
    }
  }
}

// Sum each of the 16 values v[0..15] over the warp.  Each xor level keeps half of the
// values and sends the other half to the partner, so lanes 2i and 2i + 1 end with the sum
// of value i (15 exchanges instead of 80).  Every value goes through the same xor tree
// (16, 8, 4, 2, 1), so its sum does not depend on its index.
__device__ __forceinline__ float warp_sum16(float* v, int lane) {
#pragma unroll
  for (int lvl = 0; lvl < 4; ++lvl) {
    const int half = 8 >> lvl;
    const bool up = (lane >> (4 - lvl)) & 1;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float keep = up ? v[half + i] : v[i];
      const float send = up ? v[i] : v[half + i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16 >> lvl);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

template <typename T, bool SILU>
__global__ void __launch_bounds__(512) ln_conv_kernel(LnConvParams p) {
  constexpr int VEC = Vec<T>::N, NP = VEC / 2, R = LNC_ROWS;
  extern __shared__ uint8_t smem_raw[];
  const int row_bytes = p.D * (int)sizeof(T);
  const int stage_bytes = R * row_bytes;
  const int G = p.D / VEC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, NW = blockDim.x >> 5;
  // smem: ring [nst][R rows] | partial sums [2][16][NW] fp32 | mbarriers [nst + 1]
  // 128-byte aligned by shared-space offset (pointer arithmetic on the array keeps accesses ld/st.shared)
  uint8_t* ring = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  float* red = reinterpret_cast<float*>(ring + (size_t)p.nst * stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + 2 * 16 * NW);

  const int seg = blockIdx.x;
  const int b = seg / p.segs_per_b;
  const int l0 = (seg - b * p.segs_per_b) * p.seg_len;
  const int l1 = min(l0 + p.seg_len, p.L);
  const int ntiles = (l1 - l0 + R - 1) / R;
  const T* __restrict__ x = static_cast<const T*>(p.x) + (size_t)b * p.L * p.D;
  T* __restrict__ out = static_cast<T*>(p.out) + (size_t)b * p.L * p.D;
  const float invD = 1.0f / (float)p.D;
  const int c = tid;
  const bool active = c < G;

  if (tid == 0) {
    for (int i = 0; i <= p.nst; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // tiles issued (thread 0)
  auto issue = [&](int k) {
    const int t0 = l0 + k * R;
    const int nv = min(R, l1 - t0);
    uint64_t* bar = &bars[k % p.nst];
    mbar_expect_tx(bar, (uint32_t)(nv * row_bytes));
    bulk_g2s(ring + (size_t)(k % p.nst) * stage_bytes, x + (size_t)t0 * p.D, (uint32_t)(nv * row_bytes), bar);
    issued = k + 1;
  };
  // the three rows before the segment (x rows or the halo) go to the last stage, whose first
  // tile (nst - 1) is issued only once they have been consumed; zero rows need no copy
  const bool pre_zero = (l0 == 0 && p.halo == nullptr);
  uint8_t* pre = ring + (size_t)(p.nst - 1) * stage_bytes;
  if (tid == 0) {
    if (l0 == 0 && p.halo && p.halo_flag) {
      // the peer's stores of the halo are visible once its flag is acquired; the bulk copy
      // below reads them through the async proxy.  A timed-out wait records code 43 and the
      // segment proceeds (the output is then invalid; hdc_device_error reports it).
      wait_flag(p.halo_flag, *p.halo_gen, 43);
      fence_proxy_async_global();
    }
    if (!pre_zero) {
      const T* src = l0 > 0 ? x + (size_t)(l0 - 3) * p.D : static_cast<const T*>(p.halo) + (size_t)b * 3 * p.D;
      mbar_expect_tx(&bars[p.nst], (uint32_t)(3 * row_bytes));
      bulk_g2s(pre, src, (uint32_t)(3 * row_bytes), &bars[p.nst]);
    }
    for (int k = 0; k < p.nst - 1 && k < ntiles; ++k) issue(k);
  }

  // parameters of this thread's channels, as fp32 pairs: z-space taps c0..c3, norm_w and
  // the folded bias norm_b * (c0 + c1 + c2 + c3) + cb
  uint64_t w2[NP], bb2[NP], c0[NP], c1[NP], c2[NP], c3[NP];
  {
    const int cc = active ? c : G - 1;
    float nw[VEC], nb[VEC], cb[VEC], cw[4][VEC];
    unpack16<T>(ldg16(static_cast<const T*>(p.nw) + cc * VEC), nw);
    unpack16<T>(ldg16(static_cast<const T*>(p.nb) + cc * VEC), nb);
    unpack16<T>(ldg16(static_cast<const T*>(p.cb) + cc * VEC), cb);
    const T* cwp = static_cast<const T*>(p.cw) + (size_t)cc * VEC * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f[VEC];
      unpack16<T>(ldg16(cwp + q * VEC), f);
#pragma unroll
      for (int e = 0; e < VEC; ++e) cw[(q * VEC + e) & 3][(q * VEC + e) >> 2] = f[e];
    }
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const int e0 = 2 * j, e1 = 2 * j + 1;
      w2[j] = f2_make(nw[e0], nw[e1]);
      bb2[j] = f2_make(fmaf(nb[e0], (cw[0][e0] + cw[1][e0]) + (cw[2][e0] + cw[3][e0]), cb[e0]),
                       fmaf(nb[e1], (cw[0][e1] + cw[1][e1]) + (cw[2][e1] + cw[3][e1]), cb[e1]));
      c0[j] = f2_make(cw[0][e0], cw[0][e1]);
      c1[j] = f2_make(cw[1][e0], cw[1][e1]);
      c2[j] = f2_make(cw[2][e0], cw[2][e1]);
      c3[j] = f2_make(cw[3][e0], cw[3][e1]);
    }
  }

  // shared addresses: stage s, row r, this thread's vector at ring_a + s * stage_bytes +
  // r * row_bytes + cc * 16; a lane past the last vector (D / VEC not a multiple of 32)
  // reads the last vector and stores nothing
  const uint32_t ring_a = smem_u32(ring);
  const int cc = active ? c : G - 1;

  // Reduce this thread's partial sums of a stage (`nv` valid rows) over the CTA through
  // `rb`, then finalise: lane r < 8 of every warp returns row r's mean, rstd and
  // -mean * rstd.  Contains one __syncthreads; returns the AND of every thread's `got`.
  auto tile_stats = [&](uint32_t rows_a, int nv, float* rb, bool got, float& mean, float& rs,
                        float& mrs) -> bool {
    float v[16];
    if (nv == R) row_partials<T, true>(rows_a + cc * 16, rows_a, row_bytes, R, v);
    else row_partials<T, false>(rows_a + cc * 16, rows_a, row_bytes, nv, v);
    if (!active) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
    }
    const float s = warp_sum16(v, lane);
    if ((lane & 1) == 0) rb[(lane >> 1) * NW + warp] = s;
    const bool all_ok = __syncthreads_and(got) != 0;
    float S = 0.f;
    if (lane < 16) {
      S = rb[lane * NW];
      for (int w = 1; w < NW; ++w) S += rb[lane * NW + w];
    }
    const float Sq = __shfl_down_sync(0xffffffffu, S, 8);
    mean = 0.f;
    rs = 0.f;
    mrs = 0.f;
    if (lane < R) {
      const float K = lds_elem<T>(rows_a + lane * row_bytes);
      const float m1 = S * invD;
      const float var = fmaxf(fmaf(-m1, m1, Sq * invD), 0.f);
      mean = K + m1;
      rs = rsqrtf(var + p.eps);
      mrs = -mean * rs;
    }
    return all_ok;
  };

  // conv window: W[rho & 3] holds z of row rho (relative to the segment start; rows -3..-1
  // are the preceding rows), so with 8-row tiles and the row loop unrolled every index is
  // a compile-time constant
  uint64_t W[4][NP];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < NP; ++j) W[i][j] = 0ull;  // z of a zero row is 0

  // z, conv, affine (and SiLU) of the rows of a stage; stores row r at orow + r * D
  auto conv_rows = [&](auto full, uint32_t va, T* orow, int nv, float rs, float mrs) {
    constexpr bool FULL = decltype(full)::value;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float rsr = __shfl_sync(0xffffffffu, rs, r), mrsr = __shfl_sync(0xffffffffu, mrs, r);
      if (FULL || r < nv) {
        const uint64_t rs2 = f2_make(rsr, rsr), mrs2 = f2_make(mrsr, mrsr);
        uint64_t xp[NP], o[NP];
        vec_to_f2<T>(lds16(va + r * row_bytes), xp);
#pragma unroll
        for (int j = 0; j < NP; ++j) {
          const uint64_t z = f2_fma(xp[j], rs2, mrs2);  // (x - mean) * rstd
          uint64_t a = f2_mul(z, c3[j]);
          a = f2_fma(W[(r + 3) & 3][j], c2[j], a);  // row t-1
          a = f2_fma(W[(r + 2) & 3][j], c1[j], a);  // row t-2
          a = f2_fma(W[(r + 1) & 3][j], c0[j], a);  // row t-3
          uint64_t v = f2_fma(a, w2[j], bb2[j]);
          if (SILU) {  // v * sigmoid(v) = h + h * tanh(h), h = v / 2
            const uint64_t h = f2_mul(v, f2_make(0.5f, 0.5f));
            float h0, h1, t0f, t1f;
            f2_split(h, h0, h1);
            asm("tanh.approx.f32 %0, %1;" : "=f"(t0f) : "f"(h0));
            asm("tanh.approx.f32 %0, %1;" : "=f"(t1f) : "f"(h1));
            v = f2_fma(h, f2_make(t0f, t1f), h);
          }
          o[j] = v;
          W[r & 3][j] = z;
        }
        stg16_if(orow + (size_t)r * p.D, f2_to_vec<T>(o), active);
      }
    }
  };

  bool ok = true;
  if (!pre_zero) {
    const bool got = mbar_wait(&bars[p.nst], 0, 31);
    const uint32_t pre_a = ring_a + (uint32_t)((p.nst - 1) * stage_bytes);
    float mean, rs, mrs;
    ok = tile_stats(pre_a, 3, red + 16 * NW, got, mean, rs, mrs);
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      // the same expression as the row loop, so a halo row gives the same bits
      const float rsr = __shfl_sync(0xffffffffu, rs, r), mrsr = __shfl_sync(0xffffffffu, mrs, r);
      const uint64_t rs2 = f2_make(rsr, rsr), mrs2 = f2_make(mrsr, mrsr);
      uint64_t xp[NP];
      vec_to_f2<T>(lds16(pre_a + r * row_bytes + cc * 16), xp);
#pragma unroll
      for (int j = 0; j < NP; ++j) W[r + 1][j] = f2_fma(xp[j], rs2, mrs2);
    }
  }

  int k = 0;
  for (; k < ntiles && ok; ++k) {
    const int st = k % p.nst;
    const uint32_t tile_a = ring_a + (uint32_t)(st * stage_bytes);
    const int t0 = l0 + k * R;
    const int nv = min(R, l1 - t0);
    const bool got = mbar_wait(&bars[st], (uint32_t)((k / p.nst) & 1), 32);
    float mean, rs, mrs;
    if (!tile_stats(tile_a, nv, red + (k & 1) * 16 * NW, got, mean, rs, mrs)) { ok = false; break; }
    // every thread has finished tile k - 1 (its conv came before the barrier above): refill
    // its stage with tile k + nst - 1
    if (tid == 0 && k + p.nst - 1 < ntiles) {
      fence_proxy_async_smem();  // order the generic reads of that stage before the async refill
      issue(k + p.nst - 1);
    }
    if (p.mean && warp == 0 && lane < nv) {
      p.mean[(size_t)b * p.L + t0 + lane] = __float2bfloat16_rn(mean);
      p.rstd[(size_t)b * p.L + t0 + lane] = __float2bfloat16_rn(rs);
    }
    T* orow = out + (size_t)t0 * p.D + cc * VEC;
    if (nv == R) conv_rows(std::true_type{}, tile_a + cc * 16, orow, R, rs, mrs);
    else conv_rows(std::false_type{}, tile_a + cc * 16, orow, nv, rs, mrs);
  }
  // after a timed-out wait: let this CTA's own copies in flight land (bounded) before exit
  if (!ok && tid == 0) {
    if (!pre_zero) mbar_wait(&bars[p.nst], 0, 33);
    for (int j = k; j < issued; ++j) mbar_wait(&bars[j % p.nst], (uint32_t)((j / p.nst) & 1), 33);
  }
}

template <typename T, bool SILU>
static int launch_ln_conv(LnConvParams p, int64_t B, cudaStream_t stream) {
  const int G = p.D / Vec<T>::N;
  const int threads = (G + 31) / 32 * 32;
  const int row_bytes = p.D * (int)sizeof(T);
  auto smem_of = [&](int s) {
    return (size_t)128 + (size_t)s * LNC_ROWS * row_bytes + 2 * 16 * (threads / 32) * 4 + (s + 1) * 8 + 16;
  };
  int nst = 3;
  while (smem_of(nst) > 227 * 1024 && nst > 2) --nst;
  const size_t smem = smem_of(nst);
  if (smem > 227 * 1024) return fail(HDC_E_SHAPE, "ln_conv: D=%d needs %zu bytes of shared memory", p.D, smem);
  cudaFuncSetAttribute(ln_conv_kernel<T, SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ln_conv_kernel<T, SILU>, threads, smem);
  if (occ < 1) occ = 1;
  const int64_t target = (int64_t)num_sms() * occ;
  // rounded down, so B * segs_per_b stays within one wave of resident CTAs
  int64_t segs_per_b = target / B > 0 ? target / B : 1;
  int64_t seg_len = (p.L + segs_per_b - 1) / segs_per_b;
  seg_len = ((seg_len + LNC_ROWS - 1) / LNC_ROWS) * LNC_ROWS;
  segs_per_b = (p.L + seg_len - 1) / seg_len;
  p.seg_len = (int)seg_len;
  p.segs_per_b = (int)segs_per_b;
  p.total_segs = (int)(B * segs_per_b);
  p.nst = nst;
  ln_conv_kernel<T, SILU><<<p.total_segs, threads, smem, stream>>>(p);
  return launch_status("ln_conv_kernel");
}

template <typename T>
static int ln_conv_dispatch(LnConvParams p, int64_t B, cudaStream_t stream) {
  const int G = p.D / Vec<T>::N;
  if (G <= 512)
    return p.act == HDC_ACT_SILU ? launch_ln_conv<T, true>(p, B, stream) : launch_ln_conv<T, false>(p, B, stream);
  return fail(HDC_E_SHAPE, "ln_conv: D=%d too large", p.D);
}

}  // namespace hdc

using namespace hdc;

static int ln_conv_fwd(int dtype, const void* x, const void* norm_w, const void* norm_b, const void* conv_w,
                       const void* conv_b, const void* halo, void* out, void* mean, void* rstd, int64_t B,
                       int64_t L, int64_t D, float eps, int act, const uint32_t* halo_flag,
                       const uint32_t* halo_gen, hdc_stream_t stream) {
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
  p.halo_flag = halo_flag; p.halo_gen = halo_gen;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  return dtype == HDC_F32 ? ln_conv_dispatch<float>(p, B, s) : ln_conv_dispatch<__nv_bfloat16>(p, B, s);
}

extern "C" int hdc_ln_conv_fwd(int dtype, const void* x, const void* norm_w, const void* norm_b,
                               const void* conv_w, const void* conv_b, const void* halo, void* out,
                               void* mean, void* rstd, int64_t B, int64_t L, int64_t D, float eps,
                               int act, hdc_stream_t stream) {
  return ln_conv_fwd(dtype, x, norm_w, norm_b, conv_w, conv_b, halo, out, mean, rstd, B, L, D, eps, act, nullptr,
                     nullptr, stream);
}

extern "C" int hdc_ln_conv_fwd_halo_flag(int dtype, const void* x, const void* norm_w, const void* norm_b,
                                         const void* conv_w, const void* conv_b, const void* halo, void* out,
                                         void* mean, void* rstd, int64_t B, int64_t L, int64_t D, float eps,
                                         int act, const uint32_t* halo_flag, const uint32_t* halo_gen,
                                         hdc_stream_t stream) {
  if (!halo || !halo_flag || !halo_gen) return fail(HDC_E_NULL, "ln_conv_halo_flag: halo, flag and gen required");
  return ln_conv_fwd(dtype, x, norm_w, norm_b, conv_w, conv_b, halo, out, mean, rstd, B, L, D, eps, act, halo_flag,
                     halo_gen, stream);
}
