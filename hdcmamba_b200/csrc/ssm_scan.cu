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
// Schedule: one CTA per (chunk, group of 16 channels, batch) with 16*S <= 256 threads;
// thread (j, s) scans C/S consecutive steps of channel j (16 at C 256), loading them into
// registers up front.  Segment results are combined through
// shared memory: (h_s, sum_log_s) with h = h_prev * exp(sum_log_s) + h_s.
//   pass 1 (hdc_ssm_chunk_stats): chunk statistics -> stats[b, n, 0:2ds]
//   pass 2 (hdc_ssm_scan_out):    exclusive prefix over all earlier chunks (including
//                                 n_prev chunks of earlier sequence segments),
//                                 then the outputs, written with caller strides.
#include <mutex>

#include <climits>
#include <type_traits>

#include "common.cuh"

namespace hdc {

struct SsmParams {
  const void* projs; int64_t psb, pst;
  const void* A_log;
  float* stats_w; const float* stats_r; int64_t stats_sb; int n_prev;
  // statistics read in blocks of `blk` chunks, blocks `blk_stride` floats apart (the
  // rank-major layout of gathered per-rank statistics); blk = INT_MAX: one block
  int blk; int64_t blk_stride;
  void* y; int64_t ysb, yst;
  int L, ds, C, S;
  int CG;  // channels per CTA (grid.y = ds / CG channel groups)
};

// Steps of one segment held in registers at a time.  All loads of a tile are issued before
// any arithmetic, so a segment costs one memory latency per tile instead of one per step.
constexpr int kTile = 8;

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

template <typename T>
__device__ __forceinline__ float ldnc(const T* ptr) {
  return to_f(__ldg(ptr));
}

// (log decay, input) of steps [t0, t0 + cnt) of channel j, cnt <= kTile
template <typename T>
__device__ __forceinline__ void ssm_tile(const SsmParams& p, const T* base, int j, float A, int cnt, float* ld,
                                         float* u) {
  float dt[kTile], xv[kTile], bv[kTile];
#pragma unroll
  for (int t = 0; t < kTile; ++t) {
    if (t < cnt) {
      const T* row = base + (size_t)t * p.pst;
      dt[t] = ldnc(row + j);
      xv[t] = ldnc(row + p.ds + j);
      bv[t] = ldnc(row + 2 * p.ds + j);
    }
  }
#pragma unroll
  for (int t = 0; t < kTile; ++t) {
    if (t < cnt) {
      const float dts = ssoftplus<T>(dt[t]);
      ld[t] = dts * A;
      u[t] = dts * bv[t] * xv[t];
    }
  }
}

// per-thread scan of its segment from h = 0: (h, sum_log).  With a segment of at most
// kTile steps, ld / u keep the whole segment for the output pass.
template <typename T>
__device__ __forceinline__ void ssm_segment(const SsmParams& p, const T* base, int j, float A, float* ld, float* u,
                                            float& h, float& sl) {
  const int seglen = p.C / p.S;
  h = 0.f;
  sl = 0.f;
  for (int t0 = 0; t0 < seglen; t0 += kTile) {
    const int cnt = min(kTile, seglen - t0);
    ssm_tile<T>(p, base + (size_t)t0 * p.pst, j, A, cnt, ld, u);
#pragma unroll
    for (int t = 0; t < kTile; ++t) {
      if (t < cnt) {
        sl += ld[t];
        h = h * sexp<T>(ld[t]) + u[t];
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ssm_chunk_stats_kernel(SsmParams p) {
  extern __shared__ float sh[];  // [2][S][CG]
  const int n = blockIdx.x, b = blockIdx.z;
  const int jl = threadIdx.x % p.CG, s = threadIdx.x / p.CG, j = blockIdx.y * p.CG + jl;
  const int N = p.L / p.C;
  const float A = -expf(to_f(static_cast<const T*>(p.A_log)[j]));
  const int seglen = p.C / p.S;
  const T* base = static_cast<const T*>(p.projs) + (size_t)b * p.psb + (size_t)(n * p.C + s * seglen) * p.pst;
  float ld[kTile], u[kTile], h, sl;
  ssm_segment<T>(p, base, j, A, ld, u, h, sl);
  sh[s * p.CG + jl] = h;
  sh[(p.S + s) * p.CG + jl] = sl;
  __syncthreads();
  if (s == 0) {
    float hc = 0.f, lc = 0.f;
    for (int q = 0; q < p.S; ++q) {
      hc = hc * sexp<T>(sh[(p.S + q) * p.CG + jl]) + sh[q * p.CG + jl];
      lc += sh[(p.S + q) * p.CG + jl];
    }
    float* st = p.stats_w + ((size_t)b * N + n) * 2 * p.ds;
    st[j] = bf16_round(hc);
    st[p.ds + j] = bf16_round(lc);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ssm_scan_out_kernel(SsmParams p) {
  extern __shared__ float sh[];  // [2][S][CG] + [CG] prefix
  const int n = blockIdx.x, b = blockIdx.z;
  const int jl = threadIdx.x % p.CG, s = threadIdx.x / p.CG, j = blockIdx.y * p.CG + jl;
  const float A = -expf(to_f(static_cast<const T*>(p.A_log)[j]));
  float* shG = sh + 2 * p.S * p.CG;
  const int seglen = p.C / p.S;
  const int t0 = n * p.C + s * seglen;
  const T* base = static_cast<const T*>(p.projs) + (size_t)b * p.psb + (size_t)t0 * p.pst;

  // this thread's segment first (its loads overlap the prefix below)
  float ld[kTile], u[kTile], h, sl;
  ssm_segment<T>(p, base, j, A, ld, u, h, sl);
  sh[s * p.CG + jl] = h;
  sh[(p.S + s) * p.CG + jl] = sl;
  // exclusive prefix over chunks [0, n_prev + n) -- fp32, sequential (the reference order)
  if (s == 0) {
    const int m_end = p.n_prev + n;
    float G = 0.f;
    for (int m0 = 0, blkno = 0; m0 < m_end; ++blkno) {
      const float* st = p.stats_r + (size_t)blkno * p.blk_stride + (size_t)b * p.stats_sb;
      const int m1 = min(m_end - m0, p.blk);
#pragma unroll 4
      for (int m = 0; m < m1; ++m)
        G = G * sexp<T>(st[(size_t)m * 2 * p.ds + p.ds + j]) + st[(size_t)m * 2 * p.ds + j];
      m0 += m1;
    }
    shG[jl] = bf16_round(G);
  }
  __syncthreads();
  // carry-in from earlier segments of this chunk
  float hin = 0.f, cum = 0.f;
  for (int q = 0; q < s; ++q) {
    hin = hin * sexp<T>(sh[(p.S + q) * p.CG + jl]) + sh[q * p.CG + jl];
    cum += sh[(p.S + q) * p.CG + jl];
  }
  const float G = shG[jl];
  T* yb = static_cast<T*>(p.y) + (size_t)b * p.ysb + (size_t)t0 * p.yst;
  float hh = hin;
  for (int tb = 0; tb < seglen; tb += kTile) {
    const int cnt = min(kTile, seglen - tb);
    if (seglen > kTile) ssm_tile<T>(p, base + (size_t)tb * p.pst, j, A, cnt, ld, u);
#pragma unroll
    for (int t = 0; t < kTile; ++t) {
      if (t < cnt) {
        cum += ld[t];
        hh = hh * sexp<T>(ld[t]) + u[t];
        const float yv = bf16_round(bf16_round(hh) + G * sexp<T>(cum));
        yb[(size_t)(tb + t) * p.yst + j] = from_f<T>(yv);
      }
    }
  }
}

// Channels per CTA: 16, so a chunk's channels spread over ds / 16 CTAs (one CTA per chunk
// is instruction-bound on a single SM: softplus and exp for every step of every channel).
static int ssm_group(int ds) { return ds < 16 ? ds : 16; }

// Segments per chunk: steps of C / S per thread, at least 4, at most 256 threads per CTA.
static int ssm_segments(int ds, int C) {
  const int cg = ssm_group(ds);
  int S = 1;
  while (S * 2 * cg <= 256 && C % (S * 2) == 0 && C / (S * 2) >= 4) S *= 2;
  return S;
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
  p.L = (int)L; p.ds = (int)ds; p.C = (int)C; p.S = ssm_segments((int)ds, (int)C); p.CG = ssm_group((int)ds);
  dim3 grid((unsigned)(L / C), (unsigned)(ds / p.CG), (unsigned)B);
  const size_t smem = 2 * p.S * p.CG * sizeof(float);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32) ssm_chunk_stats_kernel<float><<<grid, p.S * p.CG, smem, s>>>(p);
  else ssm_chunk_stats_kernel<__nv_bfloat16><<<grid, p.S * p.CG, smem, s>>>(p);
  return launch_status("ssm_chunk_stats_kernel");
}

static int ssm_scan_out_launch(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st, const void* A_log,
                               const float* stats, int64_t stats_sb, int64_t blk, int64_t blk_stride,
                               int64_t n_prev, void* y, int64_t y_sb, int64_t y_st, int64_t B, int64_t L,
                               int64_t ds, int64_t C, hdc_stream_t stream) {
  if (int e = ssm_check(dtype, projs, A_log, B, L, ds, C)) return e;
  if (!stats || !y) return fail(HDC_E_NULL, "ssm: null stats / y");
  SsmParams p{};
  p.projs = projs; p.psb = proj_sb; p.pst = proj_st; p.A_log = A_log; p.stats_r = stats;
  p.stats_sb = stats_sb; p.n_prev = (int)n_prev; p.y = y; p.ysb = y_sb; p.yst = y_st;
  p.blk = (int)blk; p.blk_stride = blk_stride;
  p.L = (int)L; p.ds = (int)ds; p.C = (int)C; p.S = ssm_segments((int)ds, (int)C); p.CG = ssm_group((int)ds);
  dim3 grid((unsigned)(L / C), (unsigned)(ds / p.CG), (unsigned)B);
  const size_t smem = (2 * p.S + 1) * p.CG * sizeof(float);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32) ssm_scan_out_kernel<float><<<grid, p.S * p.CG, smem, s>>>(p);
  else ssm_scan_out_kernel<__nv_bfloat16><<<grid, p.S * p.CG, smem, s>>>(p);
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

extern "C" int hdc_ssm_scan_out_blocked(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                                        const void* A_log, const float* stats, int64_t stats_sb,
                                        int64_t block_chunks, int64_t block_stride, int64_t n_prev, void* y,
                                        int64_t y_sb, int64_t y_st, int64_t B, int64_t L, int64_t ds, int64_t C,
                                        hdc_stream_t stream) {
  if (n_prev < 0 || block_chunks < 1 || block_chunks > INT_MAX)
    return fail(HDC_E_SHAPE, "ssm: n_prev=%lld block_chunks=%lld", (long long)n_prev, (long long)block_chunks);
  if (stats_sb < 0 || (B > 1 && stats_sb < block_chunks * 2 * ds) ||
      ((n_prev + (C > 0 ? L / C : 0)) > block_chunks && block_stride < B * block_chunks * 2 * ds))
    return fail(HDC_E_SHAPE, "ssm: statistics blocks overlap (stats_sb %lld, block_stride %lld)",
                (long long)stats_sb, (long long)block_stride);
  return ssm_scan_out_launch(dtype, projs, proj_sb, proj_st, A_log, stats, stats_sb, block_chunks, block_stride,
                             n_prev, y, y_sb, y_st, B, L, ds, C, stream);
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
