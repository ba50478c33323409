// GroupNorm(head) * sigmoid(gate) + concat with y_ssm, and the row LayerNorm that
// follows it (hdcmamba/model.py:274-295, 382), sm_100a.
//
// gate_cat_kernel: one warp per (token, head).  The lane holds head_dim/32 values of
// the slot row; mean and variance are warp-shuffle reductions.  The variance adds
// (bd - hd) * mean^2 for head_dim below the reference's block width bd (its padded
// lanes hold -mean when the deviations are squared, hdcmamba/model.py:290).  The
// extra warps of each CTA copy the y_ssm row.  All strides come from the caller,
// as in the reference launch (hdcmamba/model.py:377), so the shipped and the
// corrected index maps run through the same kernel.
//
// row_layernorm_kernel: one warp per row, fp32 statistics (two-pass variance),
// result in the activation dtype; optional elementwise affine (weight, bias in the
// activation dtype, as nn.LayerNorm's (x - mean) * rstd * weight + bias in fp32).
#include "common.cuh"

namespace hdc {

struct GateParams {
  const void* y_slot; int64_t s_bh, s_n, s_c; int rows;
  const void* y_ssm; int64_t ssm_b, ssm_l;
  const void* gate; int64_t g_b, g_l;
  const void* gn_w; const void* gn_b;
  void* out; int64_t o_b, o_l;
  int L, H, hd, ds, bd;
};

template <typename T>
__global__ void gate_cat_kernel(GateParams p) {
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok = blockIdx.x;
  const int b = tok / p.L, l = tok - b * p.L;
  T* out = static_cast<T*>(p.out) + (size_t)b * p.o_b + (size_t)l * p.o_l;
  for (int h = warp; h < p.H; h += warps) {
    const T* ys = static_cast<const T*>(p.y_slot) + (size_t)(b * p.H + h) * p.s_bh + (size_t)(l / p.rows) * p.s_n +
                  (size_t)(l % p.rows) * p.s_c;
    const T* gt = static_cast<const T*>(p.gate) + (size_t)b * p.g_b + (size_t)l * p.g_l + (size_t)h * p.hd;
    float v[4];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = lane + 32 * i;
      v[i] = d < p.hd ? to_f(ys[d]) : 0.f;
      sum += v[i];
    }
    const float mean = warp_sum(sum) / (float)p.hd;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = lane + 32 * i;
      if (d < p.hd) sq += (v[i] - mean) * (v[i] - mean);
    }
    const float var = (warp_sum(sq) + (float)(p.bd - p.hd) * mean * mean) / (float)p.hd;
    const float den = sqrtf(var + 1e-5f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = lane + 32 * i;
      if (d < p.hd) {
        const int c = h * p.hd + d;
        const float w = to_f(static_cast<const T*>(p.gn_w)[c]);
        const float bb = to_f(static_cast<const T*>(p.gn_b)[c]);
        const float ygn = ((v[i] - mean) / den) * w + bb;
        const float g = to_f(gt[d]);
        out[p.ds + c] = from_f<T>(bf16_round(ygn * (1.0f / (1.0f + expf(-g)))));
      }
    }
  }
  // y_ssm copy (hdcmamba/model.py:294-295)
  const T* ss = static_cast<const T*>(p.y_ssm) + (size_t)b * p.ssm_b + (size_t)l * p.ssm_l;
  for (int j = threadIdx.x; j < p.ds; j += blockDim.x) out[j] = ss[j];
}

template <typename T>
__global__ void row_layernorm_kernel(const T* in, const T* w, const T* bb, T* out, int64_t rows, int width,
                                     float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const T* r = in + row * width;
  T* o = out + row * width;
  float s = 0.f;
  for (int c = lane; c < width; c += 32) s += to_f(r[c]);
  const float mean = warp_sum(s) / (float)width;
  float q = 0.f;
  for (int c = lane; c < width; c += 32) {
    const float d = to_f(r[c]) - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) / (float)width + eps);
  for (int c = lane; c < width; c += 32) {
    float v = (to_f(r[c]) - mean) * rstd;
    if (w) v = v * to_f(w[c]) + to_f(bb[c]);
    o[c] = from_f<T>(v);
  }
}

// Vectorized variant: one warp per row, the row held in registers as 16-byte vectors
// (lane l holds vectors l, l+32, ...), so the row is read once and written once.
// Needs width % 8 == 0 (bf16), 16-byte aligned rows and width <= 8 * 32 * MAXV.
template <int MAXV>
__global__ void row_layernorm_vec_kernel(const __nv_bfloat16* in, const __nv_bfloat16* w, const __nv_bfloat16* bb,
                                         __nv_bfloat16* out, int64_t rows, int width, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const int nv = width >> 3;
  const __nv_bfloat16* r = in + row * width;
  __nv_bfloat16* o = out + row * width;
  uint4 raw[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (lane + 32 * i < nv) raw[i] = *reinterpret_cast<const uint4*>(r + (lane + 32 * i) * 8);  // may alias out
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (lane + 32 * i < nv) {
      float f[8];
      unpack16<__nv_bfloat16>(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += f[e];
    }
  }
  const float mean = warp_sum(s) / (float)width;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (lane + 32 * i < nv) {
      float f[8];
      unpack16<__nv_bfloat16>(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) q += (f[e] - mean) * (f[e] - mean);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / (float)width + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (lane + 32 * i < nv) {
      float f[8];
      unpack16<__nv_bfloat16>(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = (f[e] - mean) * rstd;
      if (w) {
        float fw[8], fb[8];
        unpack16<__nv_bfloat16>(ldg16(w + (lane + 32 * i) * 8), fw);
        unpack16<__nv_bfloat16>(ldg16(bb + (lane + 32 * i) * 8), fb);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = f[e] * fw[e] + fb[e];
      }
      stg16(o + (lane + 32 * i) * 8, pack16<__nv_bfloat16>(f));
    }
  }
}

}  // namespace hdc

using namespace hdc;

extern "C" int hdc_gate_cat_fwd(int dtype, const void* y_slot, int64_t slot_s_bh, int64_t slot_s_n,
                                int64_t slot_s_c, int64_t slot_rows, const void* y_ssm, int64_t ssm_s_b,
                                int64_t ssm_s_l, const void* gate, int64_t gate_s_b, int64_t gate_s_l,
                                const void* gn_w, const void* gn_b, void* out, int64_t out_s_b,
                                int64_t out_s_l, int64_t B, int64_t L, int64_t H, int64_t hd, int64_t ds,
                                hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "gate: dtype %d", dtype);
  if (!y_slot || !y_ssm || !gate || !gn_w || !gn_b || !out) return fail(HDC_E_NULL, "gate: null pointer");
  if (hd < 1 || hd > 128 || H < 1 || ds < 0 || B < 1 || L < 1 || slot_rows < 1 || B * L > (int64_t)INT32_MAX)
    return fail(HDC_E_SHAPE, "gate: head_dim %lld must be in [1,128]", (long long)hd);
  GateParams p{};
  p.y_slot = y_slot; p.s_bh = slot_s_bh; p.s_n = slot_s_n; p.s_c = slot_s_c; p.rows = (int)slot_rows;
  p.y_ssm = y_ssm; p.ssm_b = ssm_s_b; p.ssm_l = ssm_s_l; p.gate = gate; p.g_b = gate_s_b; p.g_l = gate_s_l;
  p.gn_w = gn_w; p.gn_b = gn_b; p.out = out; p.o_b = out_s_b; p.o_l = out_s_l;
  p.L = (int)L; p.H = (int)H; p.hd = (int)hd; p.ds = (int)ds; p.bd = (int)feature_block(hd);
  const int warps = H < 8 ? (int)H : 8;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_F32) gate_cat_kernel<float><<<(unsigned)(B * L), 32 * warps, 0, s>>>(p);
  else gate_cat_kernel<__nv_bfloat16><<<(unsigned)(B * L), 32 * warps, 0, s>>>(p);
  return launch_status("gate_cat_kernel");
}

static int row_layernorm_launch(int dtype, const void* in, const void* w, const void* b, void* out, int64_t rows,
                                int64_t width, float eps, hdc_stream_t stream) {
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "row_layernorm: dtype %d", dtype);
  if (!in || !out) return fail(HDC_E_NULL, "row_layernorm: null pointer");
  if (rows < 1 || width < 1 || width > (1 << 20)) return fail(HDC_E_SHAPE, "row_layernorm: rows/width");
  const int wpb = 8;
  const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == HDC_BF16 && width % 8 == 0 && width <= 8 * 32 * 8 && aligned16(in) && aligned16(out) &&
      (!w || (aligned16(w) && aligned16(b)))) {
    auto i = static_cast<const __nv_bfloat16*>(in);
    auto o = static_cast<__nv_bfloat16*>(out);
    auto wp = static_cast<const __nv_bfloat16*>(w);
    auto bp = static_cast<const __nv_bfloat16*>(b);
    if (width <= 8 * 32 * 4) row_layernorm_vec_kernel<4><<<grid, 32 * wpb, 0, s>>>(i, wp, bp, o, rows, (int)width, eps);
    else row_layernorm_vec_kernel<8><<<grid, 32 * wpb, 0, s>>>(i, wp, bp, o, rows, (int)width, eps);
    return launch_status("row_layernorm_vec_kernel");
  }
  if (dtype == HDC_F32)
    row_layernorm_kernel<float><<<grid, 32 * wpb, 0, s>>>(static_cast<const float*>(in), static_cast<const float*>(w),
                                                         static_cast<const float*>(b), static_cast<float*>(out), rows,
                                                         (int)width, eps);
  else
    row_layernorm_kernel<__nv_bfloat16><<<grid, 32 * wpb, 0, s>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<const __nv_bfloat16*>(w),
        static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(out), rows, (int)width, eps);
  return launch_status("row_layernorm_kernel");
}

extern "C" int hdc_row_layernorm(int dtype, const void* in, void* out, int64_t rows, int64_t width, float eps,
                                 hdc_stream_t stream) {
  return row_layernorm_launch(dtype, in, nullptr, nullptr, out, rows, width, eps, stream);
}

extern "C" int hdc_row_layernorm_affine(int dtype, const void* in, const void* weight, const void* bias, void* out,
                                        int64_t rows, int64_t width, float eps, hdc_stream_t stream) {
  if (!weight || !bias) return fail(HDC_E_NULL, "row_layernorm_affine: null weight / bias");
  return row_layernorm_launch(dtype, in, weight, bias, out, rows, width, eps, stream);
}
