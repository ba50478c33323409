// Shared pieces of the tcgen05 slot-memory kernels (slot_tc.cu, slot_mc.cu), sm_100a.
#pragma once
#include <cuda.h>

#include "slot.cuh"
#include "flag.cuh"

namespace hdc {

struct SlotTcParams {
  const void* gamma;
  const float* log_a;
  void* y;
  int64_t y_sb, y_sh, y_st;
  const float* state_in;
  float* state_out;
  float* Rseg;  // [BH][nseg][64*64]
  float* Dseg;  // [BH][nseg]
  // fused GroupNorm * sigmoid(gate) epilogue (gate == nullptr: plain y)
  const void* gate;
  int64_t g_sb, g_st;
  const void* gn_w;
  const void* gn_b;
  int L, H, hd, N, nseg, seg_len, y_vec;
  int nseg_a;  // segments computed by pass A (nseg - 1 before pass B; nseg for the state-only call)
  // four-chunk kernels (slot_mc.cu): pass A splits each output segment but the last into
  // a_split pieces of seg_len / a_split chunks, so that more CTAs share the state pass
  int a_split;
  // states of earlier sequence parts (other ranks), folded first: part s has its state at
  // prev_R + s*prev_stride + bh*4096 and its decay product at prev_D + s*prev_stride + bh
  const float* prev_R;
  const float* prev_D;
  int64_t prev_stride;
  int nprev;
  // the earlier parts' states arrive from other GPUs: the kernel waits (bounded) until every
  // flag s of wait_mask at wait_flags reaches *wait_gen before it reads them (mask 0: no wait)
  const uint32_t* wait_flags;
  uint32_t wait_mask;
  const uint32_t* wait_gen;
};

// Advance the dynamic shared-memory base to a 1024-byte boundary of its shared-space address
// (the swizzled TMA / UMMA tiles need it).  Pointer arithmetic on the shared array keeps the
// address space known to the compiler, so accesses through the result are ld/st.shared.
__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// phi(z) = elu(z) + 1 = (z > 0 ? z + 1 : exp(z)), branch-free: max(z, 0) + exp(min(z, 0))
// (exp(0) = 1 exactly, and adding +0 to exp(z) is exact)
__device__ __forceinline__ float phi_fast(float z) { return fmaxf(z, 0.f) + fast_exp(fminf(z, 0.f)); }

// phi in place on a [rows x 64] swizzled bf16 tile; columns >= hd become `pad`.
template <int NT>
__device__ __forceinline__ void prep_tile(uint8_t* tile, int rows, int hd, bool apply_phi, float pad) {
  for (int idx = threadIdx.x; idx < rows * 8; idx += NT) {
    const int row = idx >> 3, pc = idx & 7;
    const int c0 = ((pc ^ (row & 7)) << 3);
    uint4* p = reinterpret_cast<uint4*>(tile + row * 128 + pc * 16);
    if (!apply_phi && c0 + 8 <= hd) continue;
    float f[8];
    unpack16<__nv_bfloat16>(*p, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = (c0 + e < hd) ? (apply_phi ? phi_fast(f[e]) : f[e]) : pad;
    *p = pack16<__nv_bfloat16>(f);
  }
}

// phi in place on a [ROWS x 64] swizzled bf16 tile (ROWS*8 16-byte chunks split evenly over NT
// threads); columns >= hd become `pad`.  All loads are issued before any compute.
template <int NT, int ROWS, bool PHI>
__device__ __forceinline__ void prep_tile_u(uint8_t* tile, int hd, float pad) {
  constexpr int IT = ROWS * 8 / NT;
  static_assert(IT * NT == ROWS * 8, "tile chunks must split evenly");
  uint4 v[IT];
#pragma unroll
  for (int it = 0; it < IT; ++it) v[it] = reinterpret_cast<const uint4*>(tile)[threadIdx.x + it * NT];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int idx = threadIdx.x + it * NT;
    const int row = idx >> 3, pc = idx & 7;
    const int c0 = ((pc ^ (row & 7)) << 3);
    if (c0 + 8 <= hd) {  // no padding in this 16-byte chunk
      if (!PHI) continue;
      uint32_t* w = reinterpret_cast<uint32_t*>(&v[it]);
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = phi_bf2(w[i]);
      reinterpret_cast<uint4*>(tile)[idx] = v[it];
      continue;
    }
    float f[8];
    unpack16<__nv_bfloat16>(v[it], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = (c0 + e < hd) ? (PHI ? phi_fast(f[e]) : f[e]) : pad;
    reinterpret_cast<uint4*>(tile)[idx] = pack16<__nv_bfloat16>(f);
  }
}

// chunk-local cumulative log decay (per-step mode) by one warp:
//   tab[i] = c_i = sum_{t=1..i} log_a[c0+t], tab[C] = c_{C-1} + log_a[c0] (chunk decay exponent)
// The sum runs in row order, one fp32 add per row (the sequential order of the CUDA-core kernel
// and of the oracle), so the decayed keys bf16(phi(k) exp(c_{C-1} - c_j)) see the same c_j bits.
// Every lane runs the same chain on values broadcast by shuffles (no shared-memory round trip
// per row); lane 0 stores the results.
template <int CT>
__device__ __forceinline__ void chunk_cumlog_load(const float* la, int H, float* v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int e = 0; e < CT / 32; ++e) v[e] = la[(size_t)(e * 32 + lane) * H];
}
// from log_a values loaded by chunk_cumlog_load (row e * 32 + lane in v[e] of each lane)
template <int CT>
__device__ __forceinline__ void chunk_cumlog_regs(const float* v, float* tab) {
  const int lane = threadIdx.x & 31;
  float run = 0.f;
#pragma unroll
  for (int blk = 0; blk < CT / 8; ++blk) {
    float a[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = __shfl_sync(0xffffffffu, v[(blk * 8 + e) / 32], (blk * 8 + e) % 32);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (blk > 0 || e > 0) run += a[e];
      a[e] = run;
    }
    if (lane == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) tab[blk * 8 + e] = a[e];
    }
  }
  const float a0 = __shfl_sync(0xffffffffu, v[0], 0);
  if (lane == 0) tab[CT] = run + a0;
  __syncwarp();
}
template <int CT>
__device__ __forceinline__ void chunk_cumlog_warp(const float* la, int H, float* tab) {
  float v[CT / 32];
  chunk_cumlog_load<CT>(la, H, v);
  chunk_cumlog_regs<CT>(v, tab);
}

// 3-D TMA map (columns, positions, batch) over bf16 rows: `width` columns, rows `row_stride`
// elements apart, batches `batch_stride` elements apart; box 64 x box_rows x 1, 128-byte swizzle.
int slot_make_map(CUtensorMap* m, const void* base, int64_t width, int64_t L, int64_t B, int64_t row_stride,
                  int64_t batch_stride, int box_rows);

// Chunk 64 with four chunks per CTA iteration (slot_mc.cu): plain outputs (no gate epilogue,
// no earlier sequence parts), head_dim 64, a whole number of four-chunk groups.
bool slot_mc_supported(const SlotParams& p);
void slot_mc_plan(int64_t BH, int N, int* nseg, int* seg_len, int* a_split);
int slot_mc_fwd(const SlotParams& sp, int64_t B, int64_t in_sb, int64_t in_st, void* ws, cudaStream_t s);

}  // namespace hdc
