// Shared definitions of the slot-memory kernels.
#pragma once
#include "common.cuh"

namespace hdc {

struct SlotParams {
  const void* q; const void* k; const void* v; int64_t in_sb, in_st;
  const void* gamma; const float* log_a;
  void* y; int64_t y_sb, y_sh, y_st;
  const float* state_in; float* state_out;
  float* Rst;   // CUDA-core path: [BH, N, bd, bd] chunk contributions, then entering states
  float* gC;    // CUDA-core path: [BH, N] chunk decay factors
  int L, H, hd, C, rows, N, bd;
};

// Fused GroupNorm(head) * sigmoid(gate) epilogue of the tcgen05 kernel: gate element
// (b, t, h, d) at gate + b*g_sb + t*g_st + h*hd + d; gn_w / gn_b are [H*hd].
struct SlotGate {
  const void* gate; int64_t g_sb, g_st;
  const void* gn_w; const void* gn_b;
};

// phi(z) = z > 0 ? z + 1 : exp(z)  (hdcmamba/model.py:261-262)
__device__ __forceinline__ float phi(float z) { return z > 0.f ? z + 1.f : expf(z); }

template <typename T>
__device__ __forceinline__ float trnd(float v) { return store_round<T>(v); }

// States of the sequence parts before this call's (other ranks under sequence parallelism),
// folded in order into the entering state: R <- D_s R + R_s for s = 0 .. nprev-1.  Part s
// has R_s at prev_R + s*prev_stride (fp32 [B*H][64][64]) and D_s at prev_D + s*prev_stride
// (fp32 [B*H]).
struct SlotCarry {
  const float* prev_R; const float* prev_D; int64_t prev_stride; int nprev;
  // flags guarding prev_R / prev_D when they arrive from other GPUs (mask 0: no wait)
  const uint32_t* wait_flags; uint32_t wait_mask; const uint32_t* wait_gen;
};

size_t slot_simt_workspace(int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C);
int slot_simt_fwd(int dtype, SlotParams p, int64_t B, void* ws, cudaStream_t s);
size_t slot_tc_workspace(int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C);
bool slot_tc_supported(const SlotParams& p, int64_t B, int64_t in_sb, int64_t in_st);
int slot_tc_state_fwd(const SlotParams& p, int64_t B, int64_t in_sb, int64_t in_st, void* ws, float* decay_out,
                      cudaStream_t s);
int slot_tc_fwd(const SlotParams& p, const SlotGate* gate, const SlotCarry* carry, int64_t B, int64_t in_sb,
                int64_t in_st, void* ws, cudaStream_t s);

}  // namespace hdc
