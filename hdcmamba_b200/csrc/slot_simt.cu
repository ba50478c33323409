// Slot memory (chunked decayed linear attention), CUDA-core path, sm_100a.
//
// Used for fp32 activations (the reference computes fp32 dots there) and as an
// independent cross-check of the tcgen05 kernel.  Math per (batch b, head h)
// (hdcmamba/model.py:236-272), chunk n of C rows, i, j chunk-local rows:
//   phi(z)   = z > 0 ? z + 1 : exp(z); features padded to bd = max(64, pow2(hd))
//              with ones (q, k) and zeros (v), as the reference's masked lanes are
//   s_ij     = T( (phi_q_i . phi_k_j) * dmat_ij ),  j <= i      (T = activation rounding)
//   y_i      = T( sum_j s_ij v_j  +  T(phi_q_i * qdec_i) . T(R_n) )
//   R_{n+1}  = gC_n * R_n + sum_j T(phi_k_j * kdec_j)^T v_j        (fp32)
// constant decay gamma:  dmat = exp((i-j) lg), qdec = exp(i lg), kdec = exp((C-1-j) lg),
//                        gC = exp(C lg), lg = log(gamma_h)
// per-step decay log_a:  c_i = sum_{t=1..i} log_a[c0+t];  dmat = exp(c_i - c_j),
//                        qdec = exp(c_i), kdec = exp(c_{C-1} - c_j), gC = exp(c_{C-1} + log_a[c0])
//
// Passes:  (1) slot_chunk_u_kernel   U_n = sum_j T(phi_k_j kdec_j)^T v_j   -> workspace
//          (2) slot_prefix_kernel    R_n (state entering chunk n), state_out
//          (3) slot_out_kernel       y rows, 32-row blocks
#include "slot.cuh"

namespace hdc {

// chunk-local cumulative log decay c_i (per-step mode) into sh_c[0..C)
__device__ void chunk_cumlog(const SlotParams& p, int b, int h, int n, float* sh_c) {
  if (threadIdx.x == 0) {
    const float* la = p.log_a + ((size_t)b * p.L + (size_t)n * p.C) * p.H + h;
    float c = 0.f;
    sh_c[0] = 0.f;
    for (int i = 1; i < p.C; ++i) {
      c += la[(size_t)i * p.H];
      sh_c[i] = c;
    }
  }
  __syncthreads();
}

template <typename T, int BD>
__global__ void __launch_bounds__(256) slot_chunk_u_kernel(SlotParams p) {
  constexpr int OPT = BD * BD / 256;
  __shared__ float ks[32][BD], vs[32][BD], kdec[256], sh_c[256];
  const int n = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.H, h = bh - b * p.H;
  float lg = 0.f;
  if (p.log_a) {
    chunk_cumlog(p, b, h, n, sh_c);
  } else {
    lg = logf(to_f(static_cast<const T*>(p.gamma)[h]));
  }
  for (int j = threadIdx.x; j < p.rows; j += blockDim.x)
    kdec[j] = p.log_a ? expf(sh_c[p.C - 1] - sh_c[j]) : expf((float)(p.C - 1 - j) * lg);
  __syncthreads();
  const int f0 = threadIdx.x * OPT, i = f0 / BD, e0 = f0 % BD;
  float acc[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) acc[o] = 0.f;
  const T* kb = static_cast<const T*>(p.k) + (size_t)b * p.in_sb + (size_t)n * p.C * p.in_st + (size_t)h * p.hd;
  const T* vb = static_cast<const T*>(p.v) + (size_t)b * p.in_sb + (size_t)n * p.C * p.in_st + (size_t)h * p.hd;
  for (int j0 = 0; j0 < p.rows; j0 += 32) {
    for (int idx = threadIdx.x; idx < 32 * BD; idx += blockDim.x) {
      const int jj = idx / BD, d = idx % BD, j = j0 + jj;
      float kv = 0.f, vv = 0.f;
      if (j < p.rows) {
        const float kf = d < p.hd ? trnd<T>(phi(to_f(kb[(size_t)j * p.in_st + d]))) : 1.f;
        kv = trnd<T>(kf * kdec[j]);
        vv = d < p.hd ? to_f(vb[(size_t)j * p.in_st + d]) : 0.f;
      }
      ks[jj][d] = kv;
      vs[jj][d] = vv;
    }
    __syncthreads();
    for (int jj = 0; jj < 32; ++jj) {
      const float kk = ks[jj][i];
#pragma unroll
      for (int o = 0; o < OPT; ++o) acc[o] += kk * vs[jj][e0 + o];
    }
    __syncthreads();
  }
  float* U = p.Rst + ((size_t)bh * p.N + n) * BD * BD;
#pragma unroll
  for (int o = 0; o < OPT; ++o) U[f0 + o] = acc[o];
  if (threadIdx.x == 0)
    p.gC[(size_t)bh * p.N + n] = p.log_a ? expf(sh_c[p.C - 1] + p.log_a[((size_t)b * p.L + (size_t)n * p.C) * p.H + h])
                                         : expf((float)p.C * lg);
}

template <int BD>
__global__ void __launch_bounds__(256) slot_prefix_kernel(SlotParams p) {
  constexpr int OPT = BD * BD / 256;
  const int bh = blockIdx.x;
  const int f0 = threadIdx.x * OPT;
  float R[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) R[o] = p.state_in ? p.state_in[(size_t)bh * BD * BD + f0 + o] : 0.f;
  for (int m = 0; m < p.N; ++m) {
    float* slot = p.Rst + ((size_t)bh * p.N + m) * BD * BD + f0;
    const float g = p.gC[(size_t)bh * p.N + m];
#pragma unroll
    for (int o = 0; o < OPT; ++o) {
      const float u = slot[o];
      slot[o] = R[o];
      R[o] = R[o] * g + u;
    }
  }
  if (p.state_out) {
#pragma unroll
    for (int o = 0; o < OPT; ++o) p.state_out[(size_t)bh * BD * BD + f0 + o] = R[o];
  }
}

template <typename T, int BD>
__global__ void __launch_bounds__(256) slot_out_kernel(SlotParams p) {
  constexpr int RB = 32;
  constexpr int OPT = RB * BD / 256;
  extern __shared__ float smem[];
  float* qs = smem;                  // [RB][BD]
  float* qd = qs + RB * BD;          // [RB][BD]
  float* Rs = qd + RB * BD;          // [BD][BD]
  float* ks = Rs + BD * BD;          // [32][BD]
  float* vs = ks + 32 * BD;          // [32][BD]
  float* sc = vs + 32 * BD;          // [RB][33]
  float* sh_c = sc + RB * 33;        // [256]
  const int n = blockIdx.x, bh = blockIdx.y, i0 = blockIdx.z * RB;
  if (i0 >= p.rows) return;
  const int b = bh / p.H, h = bh - b * p.H;
  float lg = 0.f;
  if (p.log_a) chunk_cumlog(p, b, h, n, sh_c);
  else lg = logf(to_f(static_cast<const T*>(p.gamma)[h]));
  const size_t rowbase = (size_t)b * p.in_sb + (size_t)n * p.C * p.in_st + (size_t)h * p.hd;
  const T* qb = static_cast<const T*>(p.q) + rowbase;
  const T* kb = static_cast<const T*>(p.k) + rowbase;
  const T* vb = static_cast<const T*>(p.v) + rowbase;
  for (int idx = threadIdx.x; idx < RB * BD; idx += blockDim.x) {
    const int ii = idx / BD, d = idx % BD, i = i0 + ii;
    float qf = 0.f, qdv = 0.f;
    if (i < p.rows) {
      qf = d < p.hd ? trnd<T>(phi(to_f(qb[(size_t)i * p.in_st + d]))) : 1.f;
      const float qdec = p.log_a ? expf(sh_c[i]) : expf((float)i * lg);
      qdv = trnd<T>(qf * qdec);
    }
    qs[idx] = qf;
    qd[idx] = qdv;
  }
  const float* Rn = p.Rst + ((size_t)bh * p.N + n) * BD * BD;
  for (int idx = threadIdx.x; idx < BD * BD; idx += blockDim.x) Rs[idx] = trnd<T>(Rn[idx]);
  __syncthreads();

  const int f0 = threadIdx.x * OPT, ri = f0 / BD, e0 = f0 % BD;
  float yin[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) yin[o] = 0.f;
  const int i_last = min(i0 + RB, p.rows) - 1;
  for (int j0 = 0; j0 <= i_last; j0 += 32) {
    for (int idx = threadIdx.x; idx < 32 * BD; idx += blockDim.x) {
      const int jj = idx / BD, d = idx % BD, j = j0 + jj;
      float kf = 0.f, vv = 0.f;
      if (j < p.rows) {
        kf = d < p.hd ? trnd<T>(phi(to_f(kb[(size_t)j * p.in_st + d]))) : 1.f;
        vv = d < p.hd ? to_f(vb[(size_t)j * p.in_st + d]) : 0.f;
      }
      ks[idx] = kf;
      vs[idx] = vv;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < RB * 32; idx += blockDim.x) {
      const int ii = idx / 32, jj = idx % 32, i = i0 + ii, j = j0 + jj;
      float s = 0.f;
      if (j <= i && i < p.rows) {
        float dot = 0.f;
        for (int d = 0; d < BD; ++d) dot += qs[ii * BD + d] * ks[jj * BD + d];
        const float dm = p.log_a ? expf(sh_c[i] - sh_c[j]) : expf((float)(i - j) * lg);
        s = trnd<T>(dot * dm);
      }
      sc[ii * 33 + jj] = s;
    }
    __syncthreads();
    for (int jj = 0; jj < 32; ++jj) {
      const float s = sc[ri * 33 + jj];
#pragma unroll
      for (int o = 0; o < OPT; ++o) yin[o] += s * vs[jj * BD + e0 + o];
    }
    __syncthreads();
  }
  float yx[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) yx[o] = 0.f;
  for (int f = 0; f < BD; ++f) {
    const float qv = qd[ri * BD + f];
#pragma unroll
    for (int o = 0; o < OPT; ++o) yx[o] += qv * Rs[f * BD + e0 + o];
  }
  const int i = i0 + ri;
  if (i < p.rows) {
    T* yrow = static_cast<T*>(p.y) + (size_t)b * p.y_sb + (size_t)h * p.y_sh + (size_t)(n * p.C + i) * p.y_st;
#pragma unroll
    for (int o = 0; o < OPT; ++o)
      if (e0 + o < p.hd) yrow[e0 + o] = from_f<T>(yin[o] + yx[o]);
  }
}

template <typename T, int BD>
int slot_simt_run(SlotParams p, int64_t B, cudaStream_t s) {
  const unsigned BH = (unsigned)(B * p.H);
  slot_chunk_u_kernel<T, BD><<<dim3(p.N, BH), 256, 0, s>>>(p);
  if (int e = launch_status("slot_chunk_u_kernel")) return e;
  slot_prefix_kernel<BD><<<BH, 256, 0, s>>>(p);
  if (int e = launch_status("slot_prefix_kernel")) return e;
  const size_t smem = (size_t)(2 * 32 * BD + BD * BD + 2 * 32 * BD + 32 * 33 + 256) * sizeof(float);
  cudaFuncSetAttribute(slot_out_kernel<T, BD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  slot_out_kernel<T, BD><<<dim3(p.N, BH, (p.rows + 31) / 32), 256, smem, s>>>(p);
  return launch_status("slot_out_kernel");
}

size_t slot_simt_workspace(int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C) {
  const int64_t bd = feature_block(hd), N = L / C;
  return (size_t)(B * H * N) * (size_t)(bd * bd + 1) * sizeof(float) + 256;
}

int slot_simt_fwd(int dtype, SlotParams p, int64_t B, void* ws, cudaStream_t s) {
  const int64_t BH = B * p.H;
  p.Rst = static_cast<float*>(ws);
  p.gC = p.Rst + (size_t)BH * p.N * p.bd * p.bd;
  if (dtype == HDC_F32) {
    return p.bd == 64 ? slot_simt_run<float, 64>(p, B, s) : slot_simt_run<float, 128>(p, B, s);
  }
  return p.bd == 64 ? slot_simt_run<__nv_bfloat16, 64>(p, B, s) : slot_simt_run<__nv_bfloat16, 128>(p, B, s);
}

}  // namespace hdc
