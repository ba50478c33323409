// Recurrent single-token decode of the HdcMamba layer, sm_100a.  No counterpart in the
// reference, whose generation re-runs the whole prefix for every token.
//
// The state is that of the chunked prefill at a chunk boundary, continued one row at a
// time with the prefill's own formulas and rounding points, so that token i of a chunk
// gets row i of the chunked computation (up to fp32 summation order):
//   * LN + conv: the three previous normalised rows (fp32), shifted every step;
//   * SSM (per channel j): the chunk-local state h and summed log decay cum from the chunk
//     start, and the carry G of the chunks before it (fp32);
//       y = r(r(h) + r(G) exp(cum));  at the chunk end G <- G exp(r(cum)) + r(h), h = cum = 0
//     with r() the bf16 rounding of bf16 activations (identity for fp32);
//   * slot memory (per batch, head): the state R at the chunk start, the update U of the
//     chunk so far (sum_j k~_j^T v_j, k~_j = r(r(phi(k_j)) gamma^(C-1-j))), and the chunk's
//     phi(k) and v rows so far;
//       S_j = phi(q) . phi(k_j),  P_j = r(S_j gamma^(i-j))  (j <= i)
//       y   = r(sum_j P_j v_j + gamma^i phi(q) r(R))
//     then GroupNorm(head) * sigmoid(gate) as the fused prefill epilogue; at the chunk end
//     R <- gamma^C R + U, U = 0.
#include <type_traits>

#include "tc.cuh"

namespace hdc {

template <typename T>
__device__ __forceinline__ float rnd(float v) {
  if constexpr (std::is_same<T, float>::value) return v;
  else return bf16_round(v);
}
template <typename T>
__device__ __forceinline__ float dexp(float x) {
  if constexpr (std::is_same<T, float>::value) return expf(x);
  else return __expf(x);
}
template <typename T>
__device__ __forceinline__ float dsoftplus(float x) {
  if constexpr (std::is_same<T, float>::value) return softplus20(x);
  else return x > 20.0f ? x : __logf(1.0f + __expf(x));
}
// phi(z) = z > 0 ? z + 1 : exp(z), with the exp of the prefill path of that dtype
template <typename T>
__device__ __forceinline__ float phi_d(float z) { return z > 0.f ? z + 1.f : dexp<T>(z); }

// block-wide sum over blockDim.x threads (a multiple of 32, at most 1024)
__device__ __forceinline__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < nw; ++w) t += sh[w];
  return t;
}

// ---------------------------------------------------------------- LN + conv, one row
template <typename T>
__global__ void ln_conv_step_kernel(const T* x, const T* nw, const T* nb, const T* cw, const T* cb, float* win,
                                    T* out, int D, float eps) {
  __shared__ float sh[32];
  const int b = blockIdx.x;
  const T* xr = x + (size_t)b * D;
  float* w = win + (size_t)b * 3 * D;
  float s = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) s += to_f(xr[d]);
  const float mean = block_sum(s, sh) / (float)D;
  float q = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float c = to_f(xr[d]) - mean;
    q = fmaf(c, c, q);
  }
  const float rs = rsqrtf(block_sum(q, sh) / (float)D + eps), mrs = -mean * rs;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float n0 = fmaf(fmaf(to_f(xr[d]), rs, mrs), to_f(nw[d]), to_f(nb[d]));
    const float w3 = w[d], w2 = w[D + d], w1 = w[2 * D + d];  // rows t-3, t-2, t-1
    const float v = fmaf(w3, to_f(cw[4 * d]), fmaf(w2, to_f(cw[4 * d + 1]),
                                                 fmaf(w1, to_f(cw[4 * d + 2]), fmaf(n0, to_f(cw[4 * d + 3]), to_f(cb[d])))));
    out[(size_t)b * D + d] = from_f<T>(v);
    w[d] = w2;
    w[D + d] = w1;
    w[2 * D + d] = n0;
  }
}

// ---------------------------------------------------------------- SSM, one step
template <typename T>
__global__ void ssm_step_kernel(const T* projs, int64_t p_sb, const T* A_log, float* h, float* cum, float* G,
                                T* y, int64_t y_sb, int B, int ds, const int* pos, int C) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * ds) return;
  const bool last = *pos == C - 1;
  const int b = i / ds, j = i - b * ds;
  const T* row = projs + (size_t)b * p_sb;
  const float A = -dexp<T>(to_f(A_log[j]));
  const float dts = dsoftplus<T>(to_f(row[j]));
  const float ld = dts * A;
  const float u = dts * to_f(row[2 * ds + j]) * to_f(row[ds + j]);
  const float c = cum[i] + ld;
  const float hh = h[i] * dexp<T>(ld) + u;
  const float g = G[i];
  y[(size_t)b * y_sb + j] = from_f<T>(rnd<T>(rnd<T>(hh) + rnd<T>(g) * dexp<T>(c)));
  if (last) {  // chunk end: fold this chunk into the carry (the prefill's statistics order)
    G[i] = g * dexp<T>(rnd<T>(c)) + rnd<T>(hh);
    h[i] = 0.f;
    cum[i] = 0.f;
  } else {
    h[i] = hh;
    cum[i] = c;
  }
}

// carry G after N whole chunks from the prefill's chunk statistics [B, N, 2*ds]
__global__ void ssm_carry_kernel(const float* stats, int B, int N, int ds, float* G, int use_fast) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * ds) return;
  const int b = i / ds, j = i - b * ds;
  const float* st = stats + (size_t)b * N * 2 * ds;
  float g = 0.f;
  for (int m = 0; m < N; ++m) {
    const float dec = st[(size_t)m * 2 * ds + ds + j];
    g = g * (use_fast ? __expf(dec) : expf(dec)) + st[(size_t)m * 2 * ds + j];
  }
  G[i] = g;
}

// ---------------------------------------------------------------- slot memory, one step
// One CTA (256 threads) per (batch, head).  R, U: fp32 [64][64] per (b, h); Kc, Vc: the
// chunk's phi(k) / v rows so far, [C][64] in T per (b, h).
template <typename T>
__global__ void __launch_bounds__(256) slot_step_kernel(const T* q, const T* k, const T* v, const T* gate,
                                                        int64_t p_sb, const T* gamma, const T* gn_w, const T* gn_b,
                                                        float* R, float* U, T* Kc, T* Vc, T* out, int64_t o_sb,
                                                        int H, int hd, int C, const int* pos) {
  __shared__ float sq[64], sk[64], sv[64], sP[256], sY[64], sTab[260], sh[32];
  const int i = *pos;
  if (i < 0 || i >= C) {  // a corrupt position: record it, write nothing
    if (threadIdx.x == 0) atomicCAS(&g_dev_error, 0, 51);
    return;
  }
  const int bh = blockIdx.x, b = bh / H, h = bh - b * H;
  const int tid = threadIdx.x;
  const size_t row = (size_t)b * p_sb + (size_t)h * hd;
  float* Rb = R + (size_t)bh * 4096;
  float* Ub = U + (size_t)bh * 4096;
  T* Kb = Kc + (size_t)bh * C * 64;
  T* Vb = Vc + (size_t)bh * C * 64;
  const float lg = logf(to_f(gamma[h]));
  for (int kk = tid; kk <= C; kk += blockDim.x) sTab[kk] = expf((float)kk * lg);
  if (tid < 64) {
    const bool in = tid < hd;
    // phi and the reference's feature padding (ones for q / k, zeros for v beyond hd)
    sq[tid] = in ? rnd<T>(phi_d<T>(to_f(q[row + tid]))) : 1.f;
    sk[tid] = in ? rnd<T>(phi_d<T>(to_f(k[row + tid]))) : 1.f;
    sv[tid] = in ? to_f(v[row + tid]) : 0.f;
    Kb[(size_t)i * 64 + tid] = from_f<T>(sk[tid]);
    Vb[(size_t)i * 64 + tid] = from_f<T>(sv[tid]);
  }
  __syncthreads();
  // S_j and P_j for j <= i (row j = i comes from the fresh k / v in shared memory)
  for (int j = tid; j <= i; j += blockDim.x) {
    float s = 0.f;
    if (j == i) {
      for (int f = 0; f < 64; ++f) s = fmaf(sq[f], sk[f], s);
    } else {
      for (int f = 0; f < 64; ++f) s = fmaf(sq[f], to_f(Kb[(size_t)j * 64 + f]), s);
    }
    sP[j] = rnd<T>(s * sTab[i - j]);
  }
  __syncthreads();
  if (tid < 64) {
    const int e = tid;
    float yi = 0.f;
    for (int j = 0; j < i; ++j) yi = fmaf(sP[j], to_f(Vb[(size_t)j * 64 + e]), yi);
    yi = fmaf(sP[i], sv[e], yi);
    float yx = 0.f;
    for (int f = 0; f < 64; ++f) yx = fmaf(sq[f], rnd<T>(Rb[f * 64 + e]), yx);
    sY[e] = rnd<T>(yi + sTab[i] * yx);
  }
  __syncthreads();
  // GroupNorm over the head (padded lanes add (64 - hd) * mean^2 to the variance) * sigmoid(gate)
  float a = (tid < hd) ? sY[tid] : 0.f;
  const float mean = block_sum(a, sh) / (float)hd;
  const float dd = (tid < hd) ? sY[tid] - mean : 0.f;
  const float ssq = block_sum(dd * dd, sh);
  const float var = (ssq + (float)(64 - hd) * mean * mean) / (float)hd;
  if (tid < hd) {
    const float w = to_f(gn_w[h * hd + tid]), bb = to_f(gn_b[h * hd + tid]), g = to_f(gate[row + tid]);
    float o;
    if constexpr (std::is_same<T, float>::value) {
      // the fp32 prefill's gate kernel: division by the deviation, exact sigmoid, and the
      // reference's bf16 rounding of the gated value
      o = bf16_round((((sY[tid] - mean) / sqrtf(var + 1e-5f)) * w + bb) * (1.0f / (1.0f + expf(-g))));
    } else {  // the bf16 prefill's fused epilogue
      o = (((sY[tid] - mean) * rsqrtf(var + 1e-5f)) * w + bb) * fast_sigmoid(g);
    }
    out[(size_t)b * o_sb + (size_t)h * hd + tid] = from_f<T>(o);
  }
  // U += k~_i^T v_i; at the chunk end R <- gamma^C R + U and U = 0
  const float kd = sTab[C - 1 - i];
  const bool last = (i == C - 1);
  const float gC = sTab[C];
  for (int idx = tid; idx < 4096; idx += blockDim.x) {
    const int f = idx >> 6, e = idx & 63;
    const float u = fmaf(rnd<T>(sk[f] * kd), sv[e], Ub[idx]);
    if (last) {
      Rb[idx] = fmaf(gC, Rb[idx], u);
      Ub[idx] = 0.f;
    } else {
      Ub[idx] = u;
    }
  }
}

}  // namespace hdc

using namespace hdc;

extern "C" int hdc_ln_conv_step(int dtype, const void* x, const void* norm_w, const void* norm_b, const void* conv_w,
                                const void* conv_b, float* window, void* out, int64_t B, int64_t D, float eps,
                                hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "ln_conv_step: dtype %d", dtype);
  if (!x || !norm_w || !norm_b || !conv_w || !conv_b || !window || !out)
    return fail(HDC_E_NULL, "ln_conv_step: null pointer");
  if (B < 1 || D < 1 || D > (1 << 16)) return fail(HDC_E_SHAPE, "ln_conv_step: B=%lld D=%lld", (long long)B, (long long)D);
  const int threads = D >= 1024 ? 1024 : (int)((D + 31) / 32 * 32);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32)
    ln_conv_step_kernel<float><<<(unsigned)B, threads, 0, s>>>(
        static_cast<const float*>(x), static_cast<const float*>(norm_w), static_cast<const float*>(norm_b),
        static_cast<const float*>(conv_w), static_cast<const float*>(conv_b), window, static_cast<float*>(out),
        (int)D, eps);
  else
    ln_conv_step_kernel<__nv_bfloat16><<<(unsigned)B, threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(norm_w),
        static_cast<const __nv_bfloat16*>(norm_b), static_cast<const __nv_bfloat16*>(conv_w),
        static_cast<const __nv_bfloat16*>(conv_b), window, static_cast<__nv_bfloat16*>(out), (int)D, eps);
  return launch_status("ln_conv_step_kernel");
}

extern "C" int hdc_ssm_step(int dtype, const void* projs, int64_t proj_sb, const void* A_log, float* h, float* cum,
                            float* G, void* y, int64_t y_sb, int64_t B, int64_t ds, const int32_t* pos, int64_t C,
                            hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "ssm_step: dtype %d", dtype);
  if (!projs || !A_log || !h || !cum || !G || !y || !pos) return fail(HDC_E_NULL, "ssm_step: null pointer");
  if (B < 1 || ds < 1 || C < 1) return fail(HDC_E_SHAPE, "ssm_step: B=%lld ds=%lld", (long long)B, (long long)ds);
  const unsigned grid = (unsigned)((B * ds + 255) / 256);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32)
    ssm_step_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(projs), proj_sb,
                                                static_cast<const float*>(A_log), h, cum, G, static_cast<float*>(y),
                                                y_sb, (int)B, (int)ds, pos, (int)C);
  else
    ssm_step_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(projs), proj_sb,
                                                        static_cast<const __nv_bfloat16*>(A_log), h, cum, G,
                                                        static_cast<__nv_bfloat16*>(y), y_sb, (int)B, (int)ds, pos, (int)C);
  return launch_status("ssm_step_kernel");
}

extern "C" int hdc_ssm_carry_fwd(int dtype, const float* stats, int64_t B, int64_t N, int64_t ds, float* G,
                                 hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "ssm_carry: dtype %d", dtype);
  if (!stats || !G) return fail(HDC_E_NULL, "ssm_carry: null pointer");
  if (B < 1 || N < 0 || ds < 1) return fail(HDC_E_SHAPE, "ssm_carry: B=%lld N=%lld ds=%lld", (long long)B,
                                            (long long)N, (long long)ds);
  ssm_carry_kernel<<<(unsigned)((B * ds + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      stats, (int)B, (int)N, (int)ds, G, dtype == HDC_BF16 ? 1 : 0);
  return launch_status("ssm_carry_kernel");
}

extern "C" int hdc_slot_step(int dtype, const void* q, const void* k, const void* v, const void* gate, int64_t proj_sb,
                             const void* gamma, const void* gn_w, const void* gn_b, float* R, float* U, void* k_cache,
                             void* v_cache, void* out, int64_t out_sb, int64_t B, int64_t H, int64_t hd, int64_t C,
                             const int32_t* pos, hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "slot_step: dtype %d", dtype);
  if (!q || !k || !v || !gate || !gamma || !gn_w || !gn_b || !R || !U || !k_cache || !v_cache || !out || !pos)
    return fail(HDC_E_NULL, "slot_step: null pointer");
  if (B < 1 || H < 1 || hd < 1 || hd > 64 || C < 1 || C > 256)
    return fail(HDC_E_SHAPE, "slot_step: B=%lld H=%lld hd=%lld C=%lld (hd <= 64, C <= 256)", (long long)B,
                (long long)H, (long long)hd, (long long)C);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)(B * H);
  if (dtype == HDC_F32)
    slot_step_kernel<float><<<grid, 256, 0, s>>>(
        static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
        static_cast<const float*>(gate), proj_sb, static_cast<const float*>(gamma), static_cast<const float*>(gn_w),
        static_cast<const float*>(gn_b), R, U, static_cast<float*>(k_cache), static_cast<float*>(v_cache),
        static_cast<float*>(out), out_sb, (int)H, (int)hd, (int)C, pos);
  else
    slot_step_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
        static_cast<const __nv_bfloat16*>(v), static_cast<const __nv_bfloat16*>(gate), proj_sb,
        static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(gn_w),
        static_cast<const __nv_bfloat16*>(gn_b), R, U, static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), static_cast<__nv_bfloat16*>(out), out_sb, (int)H, (int)hd, (int)C,
        pos);
  return launch_status("slot_step_kernel");
}
