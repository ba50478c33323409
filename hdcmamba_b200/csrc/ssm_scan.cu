// Diagonal SSM chunked scan, sm_100a.
//
// Per batch b and state channel j < ds (hdcmamba/model.py:175-233):
//   dt_s = softplus20(dt), a_t = exp(dt_s * A_j), u_t = dt_s * b_t * x_t, A_j = -exp(A_log_j)
//   within chunk n:  h_t = a_t h_{t-1} + u_t  from h = 0 at the chunk start
//   chunk stats:     last_n = bf16(h at chunk end), dec_n = bf16(sum_t dt_s*A)
//   prefix:          G_0 = 0, G_{n+1} = G_n * exp(dec_n) + last_n (fp32), used as bf16(G_n)
//   output:          y_t = bf16( bf16(h_t) + bf16(G_n) * exp(cum_log_t) )
// These are the reference's rounding points (its three kernels store bf16).
//
// Schedule: one CTA per (chunk, group of 16 channels, batch) with 16*S <= 256 threads.
// The CTA stages the chunk's dt / x / b columns of its channels in shared memory with
// 16-byte loads, all in flight at once; thread (j, s) then scans C/S consecutive steps of
// channel j (16 at C 256); segment results are combined through shared memory:
// (h_s, sum_log_s) with h = h_prev * exp(sum_log_s) + h_s.  Chunks of C = 16, 32, ..., 256
// take the 16-step kernels below instead (8 channels per CTA, loads straight from global
// memory, segments summarised by their state and decay product and combined by warp
// shuffles, the output pass scanning once).
//   pass 1 (hdc_ssm_chunk_stats): chunk statistics -> stats[b, n, 0:2ds]
//   pass 2 (hdc_ssm_scan_out):    exclusive prefix over all earlier chunks (including
//                                 n_prev chunks of earlier sequence segments; folded
//                                 in S contiguous blocks, then across blocks),
//                                 then the outputs, written with caller strides.
#include <mutex>

#include <climits>
#include <type_traits>

#include "flag.cuh"

namespace hdc {

struct SsmParams {
  const void* projs; int64_t psb, pst;
  const void* A_log;
  float* stats_w; const float* stats_r; int64_t stats_sb; int n_prev;
  // statistics read in blocks of `blk` chunks, blocks `blk_stride` floats apart (the
  // rank-major layout of gathered per-rank statistics); blk = INT_MAX: one block
  int blk; int64_t blk_stride;
  void* y; int64_t ysb, yst;
  // statistics of earlier sequence parts arriving from other GPUs: the output kernel waits
  // (bounded) until every flag s of wait_mask reaches *wait_gen before it reads them
  const uint32_t* wait_flags; uint32_t wait_mask; const uint32_t* wait_gen;
  int L, ds, C, S;
  int CG;   // channels per CTA (kCD or kCG; grid.y = ds / CG channel groups)
  int vec;  // 16-byte loads of the staged columns are aligned
};

// exp / softplus: the hardware approximations (ex2 / lg2 based, as the reference's Triton
// kernels use) for bf16 activations; the accurate library functions for fp32.
template <typename T>
__device__ __forceinline__ float sexp(float x) {
  if constexpr (std::is_same<T, float>::value) return expf(x);
  else return __expf(x);
}
template <typename T>
__device__ __forceinline__ float ssoftplus(float x) {
  if constexpr (std::is_same<T, float>::value) return softplus20(x);
  else return x > 20.0f ? x : __logf(1.0f + __expf(x));
}

constexpr int kCG = 16;  // channels per CTA

// Stage the chunk's dt / x / b columns of channel group g into shared memory,
// tile[(a * C + row) * kCG + c] for a = 0 (dt), 1 (x), 2 (b): every 16-byte load of the CTA
// is in flight at once (eight per thread per round), so staging costs one memory latency.
template <typename T>
__device__ __forceinline__ void ssm_stage(const SsmParams& p, int b, int n, int g, T* tile) {
  const T* base = static_cast<const T*>(p.projs) + (size_t)b * p.psb + (size_t)n * p.C * p.pst + g * kCG;
  if (p.vec) {
    constexpr int VE = 16 / sizeof(T);   // elements per 16-byte vector
    constexpr int VPR = kCG / VE;        // vectors per row of one array
    const int nvec = p.C * 3 * VPR;
    for (int i0 = 0; i0 < nvec; i0 += 8 * (int)blockDim.x) {
      uint4 r[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k * blockDim.x + threadIdx.x;
        if (i < nvec) {
          const int v = i % VPR, a = (i / VPR) % 3, row = i / (3 * VPR);
          r[k] = ldg16(base + (size_t)row * p.pst + a * p.ds + v * VE);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k * blockDim.x + threadIdx.x;
        if (i < nvec) {
          const int v = i % VPR, a = (i / VPR) % 3, row = i / (3 * VPR);
          *reinterpret_cast<uint4*>(tile + (a * p.C + row) * kCG + v * VE) = r[k];
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < p.C * 3 * kCG; i += blockDim.x) {
      const int c = i % kCG, a = (i / kCG) % 3, row = i / (3 * kCG);
      tile[(a * p.C + row) * kCG + c] = base[(size_t)row * p.pst + a * p.ds + c];
    }
  }
}

// (log decay, input) of step `row` of channel jl from the staged tile
template <typename T>
__device__ __forceinline__ void ssm_step(const T* tile, int C, int row, int jl, float A, float& ld, float& u) {
  const float dts = ssoftplus<T>(to_f(tile[row * kCG + jl]));
  ld = dts * A;
  u = dts * to_f(tile[(2 * C + row) * kCG + jl]) * to_f(tile[(C + row) * kCG + jl]);
}

template <typename T>
__global__ void __launch_bounds__(256) ssm_chunk_stats_kernel(SsmParams p) {
  extern __shared__ float sh[];  // [2][S][kCG] partials, then the staged tile
  T* tile = reinterpret_cast<T*>(sh + 2 * p.S * kCG);
  const int n = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int jl = threadIdx.x % kCG, s = threadIdx.x / kCG, j = g * kCG + jl;
  const int N = p.L / p.C;
  const float A = -sexp<T>(to_f(static_cast<const T*>(p.A_log)[j]));
  ssm_stage<T>(p, b, n, g, tile);
  __syncthreads();
  const int seglen = p.C / p.S;
  float h = 0.f, sl = 0.f;
  for (int t = 0; t < seglen; ++t) {
    float ld, u;
    ssm_step<T>(tile, p.C, s * seglen + t, jl, A, ld, u);
    sl += ld;
    h = h * sexp<T>(ld) + u;
  }
  sh[s * kCG + jl] = h;
  sh[(p.S + s) * kCG + jl] = sl;
  __syncthreads();
  if (s == 0) {
    float hc = 0.f, lc = 0.f;
    for (int q = 0; q < p.S; ++q) {
      hc = hc * sexp<T>(sh[(p.S + q) * kCG + jl]) + sh[q * kCG + jl];
      lc += sh[(p.S + q) * kCG + jl];
    }
    float* st = p.stats_w + ((size_t)b * N + n) * 2 * p.ds;
    st[j] = bf16_round(hc);
    st[p.ds + j] = bf16_round(lc);
  }
}

// statistics (last, dec) of chunk m of batch b in the (possibly blocked) layout
__device__ __forceinline__ const float* ssm_stats_at(const SsmParams& p, int b, int m) {
  const int blk = m / p.blk;
  return p.stats_r + (size_t)blk * p.blk_stride + (size_t)b * p.stats_sb + (size_t)(m - blk * p.blk) * 2 * p.ds;
}

template <typename T>
__global__ void __launch_bounds__(256) ssm_scan_out_kernel(SsmParams p) {
  extern __shared__ float sh[];  // [4][S][kCG] partials, then the staged tile
  T* tile = reinterpret_cast<T*>(sh + 4 * p.S * kCG);
  float* pg = sh + 2 * p.S * kCG;  // prefix partials: fold of a block of earlier chunks
  float* pd = pg + p.S * kCG;      // and its summed log decay
  const int n = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int jl = threadIdx.x % kCG, s = threadIdx.x / kCG, j = g * kCG + jl;
  const float A = -sexp<T>(to_f(static_cast<const T*>(p.A_log)[j]));
  ssm_stage<T>(p, b, n, g, tile);
  if (p.wait_mask) cta_wait_flags(p.wait_flags, p.wait_mask, p.wait_gen, 45);
  // exclusive prefix over chunks [0, m_end): segment thread s folds the contiguous block
  // [m_end * s / S, m_end * (s + 1) / S) (fp32, in chunk order); the blocks are then folded
  // in order.  The split depends only on the absolute chunk index m_end, so every rank of a
  // sequence-parallel run gets the same bits as one GPU over the whole sequence.
  {
    const int m_end = p.n_prev + n;
    const int m0 = (int)((int64_t)m_end * s / p.S), m1 = (int)((int64_t)m_end * (s + 1) / p.S);
    float G = 0.f, D = 0.f;
#pragma unroll 4
    for (int m = m0; m < m1; ++m) {
      const float* st = ssm_stats_at(p, b, m);
      const float dec = st[p.ds + j];
      G = G * sexp<T>(dec) + st[j];
      D += dec;
    }
    pg[s * kCG + jl] = G;
    pd[s * kCG + jl] = D;
  }
  __syncthreads();
  const int seglen = p.C / p.S;
  float h = 0.f, sl = 0.f;
  for (int t = 0; t < seglen; ++t) {
    float ld, u;
    ssm_step<T>(tile, p.C, s * seglen + t, jl, A, ld, u);
    sl += ld;
    h = h * sexp<T>(ld) + u;
  }
  sh[s * kCG + jl] = h;
  sh[(p.S + s) * kCG + jl] = sl;
  __syncthreads();
  float G = 0.f;
  for (int q = 0; q < p.S; ++q) G = G * sexp<T>(pd[q * kCG + jl]) + pg[q * kCG + jl];
  G = bf16_round(G);
  // carry-in from earlier segments of this chunk
  float hin = 0.f, cum = 0.f;
  for (int q = 0; q < s; ++q) {
    hin = hin * sexp<T>(sh[(p.S + q) * kCG + jl]) + sh[q * kCG + jl];
    cum += sh[(p.S + q) * kCG + jl];
  }
  const int t0 = n * p.C + s * seglen;
  T* yb = static_cast<T*>(p.y) + (size_t)b * p.ysb + (size_t)t0 * p.yst;
  float hh = hin;
  for (int t = 0; t < seglen; ++t) {
    float ld, u;
    ssm_step<T>(tile, p.C, s * seglen + t, jl, A, ld, u);
    cum += ld;
    hh = hh * sexp<T>(ld) + u;
    const float yv = bf16_round(bf16_round(hh) + G * sexp<T>(cum));
    yb[(size_t)t * p.yst + j] = from_f<T>(yv);
  }
}

// ---------------------------------------------------------------------------------
// Chunks of C = 16 S steps, S = 1, 2, 4, 8 or 16 segments of kSteps = 16 steps, kCD = 8
// channels per CTA (8 S threads, ~1 KB of shared memory).  The CTAs are small enough to
// sit on an SM next to a slot-scan CTA (one per SM with ~200 KB of shared memory), so the
// SSM, launched on a side stream, runs beside the slot kernels instead of after them.
// Two thread maps over the CTA's threads:
//  * step map (jl = tid % 8, s = tid / 8): the thread loads the 16 steps of segment s of
//    channel jl straight from global memory (all 48 loads in flight at once; the 8 lanes of
//    a segment read 16 contiguous bytes per row) and scans them;
//  * segment map (c = tid / S, s = tid % S): the S segments of channel c sit in S
//    consecutive lanes, so they combine by shuffles.
// A segment is summarised by (h, E): h its state from 0 at its start, E = prod a_t its
// decay; segments combine as (h1, E1) o (h2, E2) = (h1 E2 + h2, E1 E2), with no exp.  The
// output kernel keeps each step's local (h_t, E_t) in registers, so it scans the chunk once:
//   h(step t) = hin E_t + h_t,  y_t = bf16( bf16(h) + bf16(G) Ein E_t )
// with (hin, Ein) the exclusive combine of the earlier segments of the chunk.
// ---------------------------------------------------------------------------------
constexpr int kSteps = 16;
constexpr int kCD = 8;         // channels per CTA of these kernels
constexpr int kPad = kCD + 1;  // partials [s][kPad]: both maps touch them without bank conflicts

// local scan of segment s of channel g * kCD + jl of chunk n: states h_t and decay products
// E_t of its steps, and (STATS) the summed log decay
template <typename T, bool STATS>
__device__ __forceinline__ void ssm_local16(const SsmParams& p, int b, int n, int g, int s, int jl, float A,
                                            float (&hs)[kSteps], float (&Es)[kSteps], float& sl) {
  const T* src = static_cast<const T*>(p.projs) + (size_t)b * p.psb + (size_t)(n * p.C + s * kSteps) * p.pst +
                 g * kCD + jl;
  T dt[kSteps], xv[kSteps], bv[kSteps];
#pragma unroll
  for (int t = 0; t < kSteps; ++t) {
    const T* r = src + (size_t)t * p.pst;
    dt[t] = r[0];
    xv[t] = r[p.ds];
    bv[t] = r[2 * p.ds];
  }
  float h = 0.f, E = 1.f;
  sl = 0.f;
#pragma unroll
  for (int t = 0; t < kSteps; ++t) {
    const float dts = ssoftplus<T>(to_f(dt[t]));
    const float ld = dts * A;
    const float a = sexp<T>(ld);
    h = fmaf(h, a, dts * to_f(bv[t]) * to_f(xv[t]));
    E *= a;
    if (STATS) sl += ld;
    hs[t] = h;
    Es[t] = E;
  }
}

template <typename T>
__global__ void __launch_bounds__(128) ssm_stats16_kernel(SsmParams p) {
  // hdc_ssm_scan_fwd launches the output kernel as this grid's programmatic dependent
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float sh[3 * 16 * kPad];  // [3][S][kPad] partials (h, E, summed log decay)
  const int S = p.S;
  const int n = blockIdx.x, g = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  {
    const int jl = tid % kCD, s = tid / kCD;
    const float A = -sexp<T>(to_f(static_cast<const T*>(p.A_log)[g * kCD + jl]));
    float hs[kSteps], Es[kSteps], sl;
    ssm_local16<T, true>(p, b, n, g, s, jl, A, hs, Es, sl);
    sh[s * kPad + jl] = hs[kSteps - 1];
    sh[(S + s) * kPad + jl] = Es[kSteps - 1];
    sh[(2 * S + s) * kPad + jl] = sl;
  }
  __syncthreads();
  // segment map: ordered butterfly over the S lanes of channel c (the earlier operand
  // first, so every lane of the group ends with the same bits)
  const int c = tid / S, s = tid % S;
  float h = sh[s * kPad + c], E = sh[(S + s) * kPad + c], l = sh[(2 * S + s) * kPad + c];
  for (int m = 1; m < S; m <<= 1) {
    const float h2 = __shfl_xor_sync(0xffffffffu, h, m), E2 = __shfl_xor_sync(0xffffffffu, E, m);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, m);
    h = (s & m) ? fmaf(h2, E, h) : fmaf(h, E2, h2);
    E *= E2;
    l += l2;
  }
  if (s == 0) {
    float* st = p.stats_w + ((size_t)b * (p.L / p.C) + n) * 2 * p.ds;
    st[g * kCD + c] = bf16_round(h);
    st[p.ds + g * kCD + c] = bf16_round(l);
  }
}

template <typename T>
__global__ void __launch_bounds__(128) ssm_out16_kernel(SsmParams p) {
  __shared__ float sh[2 * 16 * kPad];  // [2][S][kPad] partials
  const int S = p.S;
  const int n = blockIdx.x, g = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  // step map: this thread's 16 steps (their loads overlap the wait and the prefix below)
  const int jl = tid % kCD, s = tid / kCD;
  const float A = -sexp<T>(to_f(static_cast<const T*>(p.A_log)[g * kCD + jl]));
  float hs[kSteps], Es[kSteps], sl;
  ssm_local16<T, false>(p, b, n, g, s, jl, A, hs, Es, sl);
  // launched as the statistics kernel's programmatic dependent (hdc_ssm_scan_fwd), the loads
  // and the local scan above overlapped its end: wait for it before reading the statistics
  // (returns at once otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (p.wait_mask) cta_wait_flags(p.wait_flags, p.wait_mask, p.wait_gen, 45);
  // segment map: exclusive prefix over chunks [0, m_end) of channel c.  Lane s folds the
  // contiguous block [m_end s / S, m_end (s + 1) / S) in chunk order (fp32), then the blocks
  // fold by an ordered butterfly.  Both depend only on the absolute chunk index m_end, so a
  // sequence-parallel rank gets the same bits as one GPU over the whole sequence.
  const int c = tid / S, sc = tid % S, jc = g * kCD + c;
  float G = 0.f;
  {
    const int m_end = p.n_prev + n;
    const int m0 = (int)((int64_t)m_end * sc / S), m1 = (int)((int64_t)m_end * (sc + 1) / S);
    float D = 0.f;
#pragma unroll 4
    for (int m = m0; m < m1; ++m) {
      const float* st = ssm_stats_at(p, b, m);
      const float dec = st[p.ds + jc];
      G = fmaf(G, sexp<T>(dec), st[jc]);
      D += dec;
    }
    for (int m = 1; m < S; m <<= 1) {
      const float G2 = __shfl_xor_sync(0xffffffffu, G, m), D2 = __shfl_xor_sync(0xffffffffu, D, m);
      G = (sc & m) ? fmaf(G2, sexp<T>(D), G) : fmaf(G, sexp<T>(D2), G2);
      D += D2;
    }
    G = bf16_round(G);
  }
  sh[s * kPad + jl] = hs[kSteps - 1];
  sh[(S + s) * kPad + jl] = Es[kSteps - 1];
  __syncthreads();
  {
    // segment map: inclusive scan over the segments, then the exclusive (hin, Ein); each
    // thread overwrites only the partials it read
    float h = sh[sc * kPad + c], E = sh[(S + sc) * kPad + c];
    for (int d = 1; d < S; d <<= 1) {
      const float h2 = __shfl_up_sync(0xffffffffu, h, d, S), E2 = __shfl_up_sync(0xffffffffu, E, d, S);
      if (sc >= d) {
        h = fmaf(h2, E, h);
        E *= E2;
      }
    }
    float hin = 0.f, Ein = 1.f;
    if (S > 1) {
      hin = __shfl_up_sync(0xffffffffu, h, 1, S);
      Ein = __shfl_up_sync(0xffffffffu, E, 1, S);
    }
    if (sc == 0) {
      hin = 0.f;
      Ein = 1.f;
    }
    sh[sc * kPad + c] = hin;
    sh[(S + sc) * kPad + c] = G * Ein;
  }
  __syncthreads();
  const float hin = sh[s * kPad + jl], GE = sh[(S + s) * kPad + jl];
  T* yb = static_cast<T*>(p.y) + (size_t)b * p.ysb + (size_t)(n * p.C + s * kSteps) * p.yst + g * kCD + jl;
#pragma unroll
  for (int t = 0; t < kSteps; ++t) {
    const float hh = fmaf(hin, Es[t], hs[t]);
    yb[(size_t)t * p.yst] = from_f<T>(bf16_round(bf16_round(hh) + GE * Es[t]));
  }
}

// the 16-step kernels take C = 16 S with S a power of two up to 16
static bool ssm_fast(int64_t C) { return C == 16 || C == 32 || C == 64 || C == 128 || C == 256; }

// Channels per CTA: 16, so a chunk's channels spread over ds / 16 CTAs.
static int ssm_group(int ds) { return ds < kCG ? ds : kCG; }

// Segments per chunk: steps of C / S per thread, at least 4, at most 256 threads per CTA.
static int ssm_segments(int ds, int C) {
  const int cg = ssm_group(ds);
  int S = 1;
  while (S * 2 * cg <= 256 && C % (S * 2) == 0 && C / (S * 2) >= 4) S *= 2;
  return S;
}

// one launch of the statistics (out = false) or output kernel for the plan in p
// dependent: the output kernel directly follows this library's statistics kernel on the
// stream, so it may be a programmatic dependent launch (16-step kernels only: they wait for
// the statistics kernel before reading its results, and read nothing else it writes)
template <typename T>
static void ssm_launch(bool out, const SsmParams& p, dim3 grid, cudaStream_t s, bool dependent = false) {
  if (ssm_fast(p.C)) {  // static shared memory only
    if (out && dependent) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(p.S * p.CG);
      cfg.dynamicSmemBytes = 0;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cudaLaunchKernelEx(&cfg, ssm_out16_kernel<T>, p);
    } else if (out) {
      ssm_out16_kernel<T><<<grid, p.S * p.CG, 0, s>>>(p);
    } else {
      ssm_stats16_kernel<T><<<grid, p.S * p.CG, 0, s>>>(p);
    }
    return;
  }
  const size_t smem = (size_t)(out ? 4 : 2) * p.S * kCG * sizeof(float) + (size_t)3 * p.C * kCG * sizeof(T);
  void (*k)(SsmParams) = out ? ssm_scan_out_kernel<T> : ssm_chunk_stats_kernel<T>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k<<<grid, p.S * p.CG, smem, s>>>(p);
}

static void ssm_setup(SsmParams& p, int dtype) {
  p.S = ssm_fast(p.C) ? (int)(p.C / kSteps) : ssm_segments(p.ds, p.C);
  p.CG = ssm_fast(p.C) ? kCD : kCG;
  const size_t es = dtype == HDC_F32 ? 4 : 2;
  p.vec = ((reinterpret_cast<uintptr_t>(p.projs) & 15u) == 0 && (p.pst * es) % 16 == 0 && (p.psb * es) % 16 == 0)
              ? 1 : 0;
}

static int ssm_check(int dtype, const void* projs, const void* A_log, int64_t B, int64_t L, int64_t ds, int64_t C) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "ssm: dtype %d", dtype);
  if (!projs || !A_log) return fail(HDC_E_NULL, "ssm: null pointer");
  if (ds < 16 || ds > 256 || (ds & (ds - 1)) != 0)
    return fail(HDC_E_SHAPE, "ssm: d_state=%lld must be a power of two in [16,256]", (long long)ds);
  if (C < 1 || L < C || L % C != 0 || B < 1) return fail(HDC_E_SHAPE, "ssm: L=%lld not a multiple of C=%lld", (long long)L, (long long)C);
  return 0;
}

}  // namespace hdc

using namespace hdc;

extern "C" int hdc_ssm_chunk_stats(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                                   const void* A_log, float* stats, int64_t B, int64_t L, int64_t ds,
                                   int64_t C, hdc_stream_t stream) {
  if (int e = ssm_check(dtype, projs, A_log, B, L, ds, C)) return e;
  if (!stats) return fail(HDC_E_NULL, "ssm: null stats");
  SsmParams p{};
  p.projs = projs; p.psb = proj_sb; p.pst = proj_st; p.A_log = A_log; p.stats_w = stats;
  p.L = (int)L; p.ds = (int)ds; p.C = (int)C;
  ssm_setup(p, dtype);
  dim3 grid((unsigned)(L / C), (unsigned)(ds / p.CG), (unsigned)B);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32) ssm_launch<float>(false, p, grid, s);
  else ssm_launch<__nv_bfloat16>(false, p, grid, s);
  return launch_status("ssm_chunk_stats_kernel");
}

static int ssm_scan_out_launch(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st, const void* A_log,
                               const float* stats, int64_t stats_sb, int64_t blk, int64_t blk_stride,
                               int64_t n_prev, void* y, int64_t y_sb, int64_t y_st, int64_t B, int64_t L,
                               int64_t ds, int64_t C, hdc_stream_t stream, const uint32_t* wait_flags = nullptr,
                               uint32_t wait_mask = 0, const uint32_t* wait_gen = nullptr,
                               bool dependent = false) {
  if (int e = ssm_check(dtype, projs, A_log, B, L, ds, C)) return e;
  if (!stats || !y) return fail(HDC_E_NULL, "ssm: null stats / y");
  SsmParams p{};
  p.projs = projs; p.psb = proj_sb; p.pst = proj_st; p.A_log = A_log; p.stats_r = stats;
  p.stats_sb = stats_sb; p.n_prev = (int)n_prev; p.y = y; p.ysb = y_sb; p.yst = y_st;
  p.blk = (int)blk; p.blk_stride = blk_stride;
  p.wait_flags = wait_flags; p.wait_mask = wait_mask; p.wait_gen = wait_gen;
  p.L = (int)L; p.ds = (int)ds; p.C = (int)C;
  ssm_setup(p, dtype);
  dim3 grid((unsigned)(L / C), (unsigned)(ds / p.CG), (unsigned)B);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32) ssm_launch<float>(true, p, grid, s, dependent);
  else ssm_launch<__nv_bfloat16>(true, p, grid, s, dependent);
  return launch_status("ssm_scan_out_kernel");
}

extern "C" int hdc_ssm_scan_out(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                                const void* A_log, const float* stats, int64_t stats_sb, int64_t n_prev,
                                void* y, int64_t y_sb, int64_t y_st, int64_t B, int64_t L, int64_t ds,
                                int64_t C, hdc_stream_t stream) {
  if (n_prev < 0 || (C > 0 && stats_sb < (n_prev + L / C) * 2 * ds))
    return fail(HDC_E_SHAPE, "ssm: stats batch stride too small");
  return ssm_scan_out_launch(dtype, projs, proj_sb, proj_st, A_log, stats, stats_sb, INT_MAX, 0, n_prev, y, y_sb,
                             y_st, B, L, ds, C, stream);
}

extern "C" int hdc_ssm_scan_fwd(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st, const void* A_log,
                                float* stats, void* y, int64_t y_sb, int64_t y_st, int64_t B, int64_t L, int64_t ds,
                                int64_t C, hdc_stream_t stream) {
  if (int e = hdc_ssm_chunk_stats(dtype, projs, proj_sb, proj_st, A_log, stats, B, L, ds, C, stream)) return e;
  if (!y) return fail(HDC_E_NULL, "ssm: null y");
  return ssm_scan_out_launch(dtype, projs, proj_sb, proj_st, A_log, stats, (L / C) * 2 * ds, INT_MAX, 0, 0, y, y_sb,
                             y_st, B, L, ds, C, stream, nullptr, 0, nullptr, /*dependent=*/true);
}

extern "C" int hdc_ssm_scan_out_blocked(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                                        const void* A_log, const float* stats, int64_t stats_sb,
                                        int64_t block_chunks, int64_t block_stride, int64_t n_prev, void* y,
                                        int64_t y_sb, int64_t y_st, int64_t B, int64_t L, int64_t ds, int64_t C,
                                        const uint32_t* wait_flags, uint32_t wait_mask, const uint32_t* wait_gen,
                                        hdc_stream_t stream) {
  if (wait_mask && (!wait_flags || !wait_gen)) return fail(HDC_E_NULL, "ssm: wait_mask needs flags and gen");
  if (n_prev < 0 || block_chunks < 1 || block_chunks > INT_MAX)
    return fail(HDC_E_SHAPE, "ssm: n_prev=%lld block_chunks=%lld", (long long)n_prev, (long long)block_chunks);
  if (stats_sb < 0 || (B > 1 && stats_sb < block_chunks * 2 * ds) ||
      ((n_prev + (C > 0 ? L / C : 0)) > block_chunks && block_stride < B * block_chunks * 2 * ds))
    return fail(HDC_E_SHAPE, "ssm: statistics blocks overlap (stats_sb %lld, block_stride %lld)",
                (long long)stats_sb, (long long)block_stride);
  return ssm_scan_out_launch(dtype, projs, proj_sb, proj_st, A_log, stats, stats_sb, block_chunks, block_stride,
                             n_prev, y, y_sb, y_st, B, L, ds, C, stream, wait_flags, wait_mask, wait_gen);
}

// ---------------------------------------------------------------------------------
// Allocation-free variant of the whole chunked scan (no counterpart in the reference).
//
// Some callers cannot allocate device memory for the chunk statistics: a host that hands
// this library only the tensors it owns (for example an inference server or a plugin
// behind a foreign-function boundary with its own memory manager), or code that must not
// call cudaMalloc while the device is in a state where allocation would synchronise or
// fail.  hdc_ssm_scan_fwd_noalloc keeps the statistics in a fixed device array that the
// library reserves when it is loaded, so the caller passes only inputs and outputs.
//
//  * Capacity: kNoAllocStatsFloats fp32 values = B * (L / C) * 2 * d_state at most (4 MiB);
//    every GPU that loads the library reserves this array until the process exits.
//  * The array's device address is looked up once per device (cudaGetSymbolAddress, with
//    that device current) on the first call there; make that first call before any CUDA
//    stream capture.
//  * All calls share the one array.  The statistics kernel rewrites every value the
//    output kernel reads, so nothing needs clearing between calls, but two calls whose
//    work overlaps on the GPU (different streams without ordering) race on the array.
// ---------------------------------------------------------------------------------
namespace hdc {

constexpr int64_t kNoAllocStatsFloats = int64_t(1) << 20;
static __device__ __align__(256) float g_noalloc_stats[kNoAllocStatsFloats];

static float* noalloc_stats_ptr(int* err) {
  static std::mutex mu;
  static float* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = fail(HDC_E_SHAPE, "ssm_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_stats);
    if (e != cudaSuccess || ptr == nullptr) {
      *err = fail((int)e ? (int)e : HDC_E_NULL, "ssm_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = static_cast<float*>(ptr);
  }
  return cache[dev];
}

}  // namespace hdc

extern "C" int64_t hdc_ssm_noalloc_capacity(void) { return hdc::kNoAllocStatsFloats; }

extern "C" int hdc_ssm_scan_fwd_noalloc(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                                        const void* A_log, void* y, int64_t y_sb, int64_t y_st, int64_t B,
                                        int64_t L, int64_t ds, int64_t C, hdc_stream_t stream) {
  if (int e = ssm_check(dtype, projs, A_log, B, L, ds, C)) return e;
  if (!y) return fail(HDC_E_NULL, "ssm_noalloc: null y");
  const int64_t need = B * (L / C) * 2 * ds;
  if (need > kNoAllocStatsFloats)
    return fail(HDC_E_WORKSPACE, "ssm_noalloc: B*(L/C)*2*d_state = %lld exceeds the fixed capacity %lld",
                (long long)need, (long long)kNoAllocStatsFloats);
  int err = 0;
  float* stats = noalloc_stats_ptr(&err);
  if (!stats) return err;
  if (int e = hdc_ssm_chunk_stats(dtype, projs, proj_sb, proj_st, A_log, stats, B, L, ds, C, stream)) return e;
  return hdc_ssm_scan_out(dtype, projs, proj_sb, proj_st, A_log, stats, (L / C) * 2 * ds, 0, y, y_sb, y_st, B, L, ds,
                          C, stream);
}
