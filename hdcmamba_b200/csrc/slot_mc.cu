// Slot memory scan at chunk 64 with four chunks per CTA iteration (tcgen05, bf16, head_dim 64),
// sm_100a.  Same math and rounding points as the other tcgen05 slot kernels (the chunked
// decayed linear attention of _slot_all_fused, hdcmamba/model.py:236-272, and its per-step
// decay generalisation); only the schedule differs.
//
// At chunk 64 one chunk carries little work per phase: 64 rows of S, P, Y and a 64 x 64 state
// update.  Walking one chunk per iteration leaves every phase latency-bound (a TMA round trip,
// a tensor-core round trip and a CTA barrier per step).  Here a CTA takes a group of G = 4
// consecutive chunks per iteration (256 rows of q, k, v in one 32 KB tile each) and runs each
// phase for all four chunks at once, with separate tensor-memory accumulators per chunk:
//
//   TMEM (512 columns): chunk x of the group has S_x, then Y_x, in [128x, 128x + 64) and
//   U_x = k~_x^T V_x in [128x + 64, 128x + 128); M = 64 products (rows 16q + l in lanes
//   32q + l, l < 16).
//
// Per group (pass B, slot_mc_out_kernel):
//   phi(K), phi(Q) in place -> S_x = phi(Q_x) phi(K_x)^T  -> k~_x, Qs_x in place, P_x to smem
//   -> U_x and P_x V_x -> the state entering each chunk, R_{x+1} = gC_x R_x + U_x (fp32, in
//   registers; bf16(R_x) into the P buffer, which is free again) -> Y_x += Qs_x bf16(R_x)
//   -> y = bf16(Y_x) stored.
// Pass A (slot_mc_state_kernel) computes each segment's local state from zero the same way
// (k~_x in place, U_x, the fold), for the segments before the last.
// Every wait is bounded (tc.cuh) and reports through hdc_device_error.
#include "slot_tc.cuh"

namespace hdc {
namespace mc {
constexpr int CT = 64, G = 4, ROWS = CT * G, NT = 512;
constexpr int TILE = ROWS * 128;  // one [256 x 64] bf16 tile, 128-byte swizzle
constexpr int CHUNK = CT * 128;   // one chunk's rows inside a tile
constexpr int TABN = CT + 4;      // one chunk's decay table (CT + 1 entries used)
constexpr size_t SMEM_A = 1024 + 4 * TILE + 2 * G * TABN * 4 + 3 * 8 + 16;
constexpr size_t SMEM_B = 1024 + 6 * TILE + 2 * G * TABN * 4 + 6 * 8 + 16;
// Pass B loads chunk x's Q rows permuted in 16-row blocks: tile rows [16 q, 16 q + 16) of the
// chunk (TMEM lane quarter q of its M = 64 accumulators) hold chunk rows of block (q + x) mod 4.
// The causal P work of a row block grows 1 : 2 : 3 : 4 with the block, and lane quarter q is
// read only by the warps of one SM sub-partition, so over the four chunks of a group every
// sub-partition gets the same P work.  Chunk row of tile row r (0 <= r < CT) of chunk x:
__host__ __device__ constexpr int q_chunk_row(int x, int r) { return ((((r >> 4) + x) & 3) << 4) | (r & 15); }
}  // namespace mc

// Decay table of chunk x of group g for this (b, h): per-step, c_i and the chunk decay
// exponent, in one of two buffers of G tables (warp x of the first G warps fills table x of
// the next group while this one is processed); constant gamma, gamma^k for k <= CT (one table).
__device__ __forceinline__ const float* mc_tab(const float* sTab, bool perstep, int g, int x) {
  return sTab + (perstep ? ((g & 1) * mc::G + x) * mc::TABN : 0);
}
__device__ __forceinline__ float* mc_tab_w(float* sTab, int g, int x) {
  return sTab + ((g & 1) * mc::G + x) * mc::TABN;
}
// log_a of chunk x of group g (rows n0 + G g + x), element (b, t, h) at (b L + t) H + h
__device__ __forceinline__ const float* mc_log_a(const SlotTcParams& p, int b, int h, int n0, int g, int x) {
  return p.log_a + ((size_t)b * p.L + (size_t)(n0 + g * mc::G + x) * mc::CT) * p.H + h;
}

// ---------------------------------------------------------------------------------
// Pass A: local state of each segment before the last (from zero) and its decay product.
// ---------------------------------------------------------------------------------
template <bool PERSTEP>
__global__ void __launch_bounds__(mc::NT, 1)
    slot_mc_state_kernel(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV,
                         SlotTcParams p) {
  using namespace mc;
  // the output kernel (launched as this grid's programmatic dependent) may start its CTAs as
  // this grid's CTAs exit; it waits for this grid before it reads the states
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  // stage st: K at base + 2 st TILE, V right after it
  float* sTab = reinterpret_cast<float*>(base + 4 * TILE);          // [2][G][TABN]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sTab + 2 * G * TABN);  // [0], [1] stage loads, [2] products
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, cgrp = warp >> 2;
  // piece `seg` of this (batch, head): chunks [seg * len, (seg + 1) * len), len = seg_len / a_split
  const int bh = blockIdx.x / p.nseg_a, seg = blockIdx.x - bh * p.nseg_a;
  const int b = bh / p.H, h = bh - b * p.H;
  const int len = p.seg_len / p.a_split;
  const int n0 = seg * len, n1 = min(p.N, n0 + len);
  const int ngroups = (n1 - n0) / G;

  if (warp == 0) {
    tmem_alloc(sTmem, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    tma_prefetch_map(&mapK);
    tma_prefetch_map(&mapV);
  }
  if (!PERSTEP) {
    const float lg = logf(__bfloat162float(static_cast<const __nv_bfloat16*>(p.gamma)[h]));
    for (int k = tid; k <= CT; k += NT) sTab[k] = expf((float)k * lg);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tU = *sTmem + ((uint32_t)(quarter * 32) << 16);
  constexpr uint32_t idU = idesc_bf16_f32(64, 64, true, true);

  float R[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) R[e] = 0.f;
  float D = 1.f;
  uint32_t fph = 0, mph = 0;
  int pending = 0;  // thread 0: bit st set while stage st has loads in flight
  bool ok = true;
  auto issue = [&](int g, int st) {
    uint8_t* sK = base + st * 2 * TILE;
    const int row = (n0 + g * G) * CT;
    mbar_expect_tx(&bars[st], 2 * TILE);
    tma_load_3d(sK, &mapK, h * p.hd, row, b, &bars[st]);
    tma_load_3d(sK + TILE, &mapV, h * p.hd, row, b, &bars[st]);
    pending |= 1 << st;
  };
  if (tid == 0) {
    if (ngroups > 0) issue(0, 0);
    if (ngroups > 1) issue(1, 1);
  }
  // per-step: tables of group 0 now; each later group's log_a is loaded a group ahead
  float la_next[CT / 32];
  if (PERSTEP) {
    if (warp < G && ngroups > 0) chunk_cumlog_warp<CT>(mc_log_a(p, b, h, n0, 0, warp), p.H, mc_tab_w(sTab, 0, warp));
    __syncthreads();
  }
  for (int g = 0; g < ngroups; ++g) {
    const int st = g & 1;
    uint8_t* sK = base + st * 2 * TILE;
    uint8_t* sV = sK + TILE;
    if (PERSTEP && warp < G && g + 1 < ngroups) chunk_cumlog_load<CT>(mc_log_a(p, b, h, n0, g + 1, warp), p.H, la_next);
    if (!mbar_wait_warp(&bars[st], (fph >> st) & 1u, 71)) { ok = false; break; }
    fph ^= 1u << st;
    if (tid == 0) pending &= ~(1 << st);
    // k~ = bf16(bf16(phi(k)) kdec_j) in place, four 16-byte pieces per thread
    {
      uint4 kv[ROWS * 8 / NT];
#pragma unroll
      for (int it = 0; it < ROWS * 8 / NT; ++it) kv[it] = reinterpret_cast<const uint4*>(sK)[tid + it * NT];
#pragma unroll
      for (int it = 0; it < ROWS * 8 / NT; ++it) {
        const int idx = tid + it * NT, row = idx >> 3, x = row >> 6, i = row & (CT - 1);
        const float* T = mc_tab(sTab, PERSTEP, g, x);
        const float kd = PERSTEP ? fast_exp(T[CT - 1] - T[i]) : T[CT - 1 - i];
        const uint64_t kd2 = f2_make(kd, kd);
        uint32_t* w = reinterpret_cast<uint32_t*>(&kv[it]);
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = f2_to_bf2(f2_mul(bf2_to_f2(phi_bf2(w[e])), kd2));
        reinterpret_cast<uint4*>(sK)[idx] = kv[it];
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int x = 0; x < G; ++x)
#pragma unroll
        for (int kk = 0; kk < CT / 16; ++kk)
          umma_bf16(*sTmem + 64 * x, sdesc_sw128(smem_u32(sK) + x * CHUNK + kk * 2048, 0, 1024),
                    sdesc_sw128(smem_u32(sV) + x * CHUNK + kk * 2048, 0, 1024), idU, kk > 0 ? 1u : 0u);
      umma_commit(&bars[2]);
    }
    if (!mbar_wait_warp(&bars[2], mph, 72)) { ok = false; break; }
    mph ^= 1;
    tc_fence_after();
    if (tid == 0 && g + 2 < ngroups) issue(g + 2, st);  // this stage's products are done
    // fold the group's chunks in order: R <- gC_x R + U_x
    float u[G][16];
    tmem_ld16x2(tU + cgrp * 16, tU + 64 + cgrp * 16, u[0], u[1]);
    tmem_ld16x2(tU + 128 + cgrp * 16, tU + 192 + cgrp * 16, u[2], u[3]);
#pragma unroll
    for (int x = 0; x < G; ++x) {
      const float* T = mc_tab(sTab, PERSTEP, g, x);
      const float gC = PERSTEP ? fast_exp(T[CT]) : T[CT];
#pragma unroll
      for (int e = 0; e < 16; ++e) R[e] = fmaf(R[e], gC, u[x][e]);
      D *= gC;
    }
    if (PERSTEP && warp < G && g + 1 < ngroups) chunk_cumlog_regs<CT>(la_next, mc_tab_w(sTab, g + 1, warp));
    // every thread's TMEM and table reads are done before the next group's products / tables
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (ok && lane < 16) {
    const int f = quarter * 16 + lane;
    float* dst = p.Rseg + ((size_t)bh * p.nseg_a + seg) * 4096 + f * 64 + cgrp * 16;
#pragma unroll
    for (int e = 0; e < 16; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(R[e], R[e + 1], R[e + 2], R[e + 3]);
  }
  if (ok && tid == 0) p.Dseg[(size_t)bh * p.nseg_a + seg] = D;
  // after a timed-out wait: let this CTA's own loads in flight land (bounded) before exit
  if (!ok && tid == 0) {
    if (pending & 1) mbar_wait(&bars[0], fph & 1u, 73);
    if (pending & 2) mbar_wait(&bars[1], (fph >> 1) & 1u, 73);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(*sTmem, 256);
}

// ---------------------------------------------------------------------------------
// Pass B: outputs.  Entering state = state_in and the earlier segments' local states,
// folded; then the groups of this segment in order.
// ---------------------------------------------------------------------------------
template <bool PERSTEP>
__global__ void __launch_bounds__(mc::NT, 1)
    slot_mc_out_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                       const __grid_constant__ CUtensorMap mapV, SlotTcParams p) {
  using namespace mc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  // stage st: K at base + 2 st TILE, Q right after it; V at 4 TILE; P / R of the group at 5 TILE
  uint8_t* sV = base + 4 * TILE;
  uint8_t* sPR = base + 5 * TILE;
  float* sTab = reinterpret_cast<float*>(base + 6 * TILE);       // [2][G][TABN]
  // mbarriers: [0], [1] K + Q of a stage, [2] V, [3] S products, [4] U and P V, [5] Qs R
  uint64_t* bars = reinterpret_cast<uint64_t*>(sTab + 2 * G * TABN);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + 6);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, wg = warp >> 2;
  const int bh = blockIdx.x / p.nseg, seg = blockIdx.x - bh * p.nseg;
  const int b = bh / p.H, h = bh - b * p.H;
  const int n0 = seg * p.seg_len, n1 = min(p.N, n0 + p.seg_len);
  const int ngroups = (n1 - n0) / G;
  const bool f_valid = lane < 16;  // this lane holds row f_row of every M = 64 product
  const int f_row = quarter * 16 + lane;
  const int e0 = wg * 16;          // accumulator columns [e0, e0 + 16)

  if (warp == 0) {
    tmem_alloc(sTmem, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    tma_prefetch_map(&mapQ);
    tma_prefetch_map(&mapK);
    tma_prefetch_map(&mapV);
  }
  if (!PERSTEP) {
    const float lg = logf(__bfloat162float(static_cast<const __nv_bfloat16*>(p.gamma)[h]));
    for (int k = tid; k <= CT; k += NT) sTab[k] = expf((float)k * lg);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  const uint32_t tL = tmem + ((uint32_t)(quarter * 32) << 16);
  constexpr uint32_t idS = idesc_bf16_f32(64, 64, false, false);
  constexpr uint32_t idPV = idesc_bf16_f32(64, 64, false, true);
  constexpr uint32_t idU = idesc_bf16_f32(64, 64, true, true);

  int pending = 0;  // thread 0: bits 0, 1 K + Q stages, bit 2 V in flight
  auto issue_kq = [&](int g, int st) {
    uint8_t* sK = base + st * 2 * TILE;
    const int row = (n0 + g * G) * CT;
    mbar_expect_tx(&bars[st], 2 * TILE);
    tma_load_3d(sK, &mapK, h * p.hd, row, b, &bars[st]);
    // Q in 16-row boxes, each chunk's row blocks permuted (q_chunk_row)
#pragma unroll
    for (int j = 0; j < ROWS / 16; ++j)
      tma_load_3d(sK + TILE + j * 16 * 128, &mapQ, h * p.hd, row + (j >> 2) * CT + q_chunk_row(j >> 2, (j & 3) * 16),
                  b, &bars[st]);
    pending |= 1 << st;
  };
  auto issue_v = [&](int g) {
    mbar_expect_tx(&bars[2], TILE);
    tma_load_3d(sV, &mapV, h * p.hd, (n0 + g * G) * CT, b, &bars[2]);
    pending |= 4;
  };
  if (tid == 0) {
    if (ngroups > 0) {
      issue_kq(0, 0);
      issue_v(0);
    }
    if (ngroups > 1) issue_kq(1, 1);
  }

  // pass A's states: when this kernel was launched as its programmatic dependent, the setup and
  // the first loads above ran while it was finishing; wait for it here (returns at once
  // otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // entering state: state_in, then the local states of pass A's pieces before this segment
  // (fp32; lanes < 16 hold row f_row, columns [e0, e0 + 16))
  float Rr[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) Rr[e] = 0.f;
  if (f_valid) {
    if (p.state_in) {
      const float4* src = reinterpret_cast<const float4*>(p.state_in + (size_t)bh * 4096 + f_row * 64 + e0);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float4 v = src[e];
        Rr[4 * e] = v.x; Rr[4 * e + 1] = v.y; Rr[4 * e + 2] = v.z; Rr[4 * e + 3] = v.w;
      }
    }
#pragma unroll 4
    for (int s = 0; s < seg * p.a_split; ++s) {
      const float Ds = p.Dseg[(size_t)bh * p.nseg_a + s];
      const float4* src =
          reinterpret_cast<const float4*>(p.Rseg + ((size_t)bh * p.nseg_a + s) * 4096 + f_row * 64 + e0);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float4 v = src[e];
        Rr[4 * e] = Ds * Rr[4 * e] + v.x;
        Rr[4 * e + 1] = Ds * Rr[4 * e + 1] + v.y;
        Rr[4 * e + 2] = Ds * Rr[4 * e + 2] + v.z;
        Rr[4 * e + 3] = Ds * Rr[4 * e + 3] + v.w;
      }
    }
  }

  uint32_t kqph = 0, vph = 0, sph = 0, aph = 0, yph = 0;
  bool ok = true;
  // phi of a stage's K and Q in place once its loads landed
  auto prep_stage = [&](int st) -> bool {
    if (!mbar_wait_warp(&bars[st], (kqph >> st) & 1u, 74)) return false;
    kqph ^= 1u << st;
    if (tid == 0) pending &= ~(1 << st);
    prep_tile_u<NT, ROWS, true>(base + st * 2 * TILE, 64, 1.f);
    prep_tile_u<NT, ROWS, true>(base + st * 2 * TILE + TILE, 64, 1.f);
    return true;
  };
  // group 0: phi and (per-step) tables now; each later group's are formed while the previous
  // group's U and P V products run, with its log_a loaded a group ahead
  float la_next[CT / 32];
  if (ngroups > 0) {
    if (PERSTEP && warp < G) chunk_cumlog_warp<CT>(mc_log_a(p, b, h, n0, 0, warp), p.H, mc_tab_w(sTab, 0, warp));
    ok = prep_stage(0);
  }
  for (int g = 0; g < ngroups && ok; ++g) {
    const int st = g & 1;
    uint8_t* sK = base + st * 2 * TILE;
    uint8_t* sQ = sK + TILE;
    if (PERSTEP && warp < G && g + 1 < ngroups) chunk_cumlog_load<CT>(mc_log_a(p, b, h, n0, g + 1, warp), p.H, la_next);
    // phi(K), phi(Q) and the tables of this group are in place
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- S_x = phi(Q_x) phi(K_x)^T
    if (tid == 0) {
#pragma unroll
      for (int x = 0; x < G; ++x)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tmem + 128 * x, sdesc_sw128(smem_u32(sQ) + x * CHUNK + k * 32, 16, 1024),
                    sdesc_sw128(smem_u32(sK) + x * CHUNK + k * 32, 16, 1024), idS, k > 0 ? 1u : 0u);
      umma_commit(&bars[3]);
    }
    if (!mbar_wait_warp(&bars[3], sph, 75)) { ok = false; break; }
    sph ^= 1;
    tc_fence_after();
    // ---- k~ = bf16(phi(k) kdec_j), Qs = bf16(phi(q) qdec_i) in place (the S products are done
    // with sK / sQ; the reference rounds the q-decayed queries, hdcmamba/model.py:267-268)
    {
      constexpr int IT = ROWS * 8 / NT;
      uint4 kv[IT], qv[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        kv[it] = reinterpret_cast<const uint4*>(sK)[tid + it * NT];
        qv[it] = reinterpret_cast<const uint4*>(sQ)[tid + it * NT];
      }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = tid + it * NT, row = idx >> 3, x = row >> 6, i = row & (CT - 1);
        const float* T = mc_tab(sTab, PERSTEP, g, x);
        const int iq = q_chunk_row(x, i);  // chunk row of Q tile row `row`
        const float kd = PERSTEP ? fast_exp(T[CT - 1] - T[i]) : T[CT - 1 - i];
        const float qd = PERSTEP ? fast_exp(T[iq]) : T[iq];
        const uint64_t kd2 = f2_make(kd, kd), qd2 = f2_make(qd, qd);
        uint32_t* wk = reinterpret_cast<uint32_t*>(&kv[it]);
        uint32_t* wq = reinterpret_cast<uint32_t*>(&qv[it]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          wk[e] = f2_to_bf2(f2_mul(bf2_to_f2(wk[e]), kd2));
          wq[e] = f2_to_bf2(f2_mul(bf2_to_f2(wq[e]), qd2));
        }
        reinterpret_cast<uint4*>(sK)[idx] = kv[it];
        reinterpret_cast<uint4*>(sQ)[idx] = qv[it];
      }
    }
    // ---- P_x = bf16(mask(S_x) decay): columns [e0, e0 + 16) of every chunk -> sPR.  The M = 64
    // accumulators fill TMEM lanes 0-15 of each quarter, so the two half-warps split the
    // columns: lanes 16-31 take columns 8-15 of the row that lane - 16 read (tile row
    // quarter * 16 + lane % 16, chunk row q_chunk_row(x, tile row)).
    {
      float sv[G][16];
      tmem_ld16x2(tL + e0, tL + 128 + e0, sv[0], sv[1]);
      tmem_ld16x2(tL + 256 + e0, tL + 384 + e0, sv[2], sv[3]);
      const int hl = lane >> 4, prow = quarter * 16 + (lane & 15);
#pragma unroll
      for (int x = 0; x < G; ++x) {
        const int qb = (quarter + x) & 3;  // chunk row block of this lane quarter
        const int i = qb * 16 + (lane & 15);
        float v[8];
        if (wg <= qb) {  // some column of the piece is at or below the diagonal of these rows
          float w[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float up = __shfl_up_sync(0xffffffffu, sv[x][8 + e], 16);
            w[e] = hl ? up : sv[x][e];
          }
          const float* T = mc_tab(sTab, PERSTEP, g, x);
          const float ci = PERSTEP ? T[i] : 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = e0 + 8 * hl + e;
            const float dm = j <= i ? (PERSTEP ? fast_exp(ci - T[j]) : T[i - j]) : 0.f;
            v[e] = j <= i ? w[e] * dm : 0.f;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = 0.f;
        }
        *reinterpret_cast<uint4*>(sPR + x * CHUNK + sw128_chunk(prow, (e0 >> 3) + hl)) = pack16<__nv_bfloat16>(v);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- U_x = k~_x^T V_x and Y_x = P_x V_x
    if (tid == 0) {
      if (mbar_wait(&bars[2], vph, 76)) {
        pending &= ~4;
        tc_fence_after();
#pragma unroll
        for (int x = 0; x < G; ++x) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + 128 * x + 64, sdesc_sw128(smem_u32(sK) + x * CHUNK + kk * 2048, 0, 1024),
                      sdesc_sw128(smem_u32(sV) + x * CHUNK + kk * 2048, 0, 1024), idU, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + 128 * x, sdesc_sw128(smem_u32(sPR) + x * CHUNK + kk * 32, 16, 1024),
                      sdesc_sw128(smem_u32(sV) + x * CHUNK + kk * 16 * 128, 0, 1024), idPV, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[4]);
      }
    }
    vph ^= 1;
    // meanwhile: the next group's phi and tables (its stage's loads were issued a group ago)
    if (g + 1 < ngroups) {
      if (PERSTEP && warp < G) chunk_cumlog_regs<CT>(la_next, mc_tab_w(sTab, g + 1, warp));
      if (!prep_stage(st ^ 1)) { ok = false; break; }
    }
    if (!mbar_wait_warp(&bars[4], aph, 77)) { ok = false; break; }
    aph ^= 1;
    tc_fence_after();
    if (tid == 0 && g + 1 < ngroups) issue_v(g + 1);  // V is free
    // ---- the state entering each chunk of the group: bf16(R_x) -> sPR (free again), then
    // R <- gC_x R + U_x (fp32)
    {
      float u[G][16];
      tmem_ld16x2(tL + 64 + e0, tL + 192 + e0, u[0], u[1]);
      tmem_ld16x2(tL + 320 + e0, tL + 448 + e0, u[2], u[3]);
      if (f_valid) {
#pragma unroll
        for (int x = 0; x < G; ++x) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
            *reinterpret_cast<uint4*>(sPR + x * CHUNK + sw128_chunk(f_row, (e0 >> 3) + c)) =
                pack16<__nv_bfloat16>(&Rr[c * 8]);
          const float* T = mc_tab(sTab, PERSTEP, g, x);
          const float gC = PERSTEP ? fast_exp(T[CT]) : T[CT];
#pragma unroll
          for (int e = 0; e < 16; ++e) Rr[e] = fmaf(Rr[e], gC, u[x][e]);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- Y_x += Qs_x bf16(R_x)
    if (tid == 0) {
#pragma unroll
      for (int x = 0; x < G; ++x)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tmem + 128 * x, sdesc_sw128(smem_u32(sQ) + x * CHUNK + k * 32, 16, 1024),
                    sdesc_sw128(smem_u32(sPR) + x * CHUNK + k * 2048, 0, 1024), idPV, 1u);
      umma_commit(&bars[5]);
    }
    if (!mbar_wait_warp(&bars[5], yph, 78)) { ok = false; break; }
    yph ^= 1;
    tc_fence_after();
    if (tid == 0 && g + 2 < ngroups) issue_kq(g + 2, st);  // this stage's K and Q are free
    // ---- y = bf16(Y_x): staged in sPR (free after the Qs R products, 128-byte swizzled rows),
    // then written out with 16-byte stores, eight threads per 128-byte row
    {
      float yv[G][16];
      tmem_ld16x2(tL + e0, tL + 128 + e0, yv[0], yv[1]);
      tmem_ld16x2(tL + 256 + e0, tL + 384 + e0, yv[2], yv[3]);
      if (p.y_vec) {
        if (f_valid) {
#pragma unroll
          for (int x = 0; x < G; ++x)
#pragma unroll
            for (int c = 0; c < 2; ++c)
              *reinterpret_cast<uint4*>(sPR + sw128_chunk(x * CT + q_chunk_row(x, f_row), (e0 >> 3) + c)) =
                  pack16<__nv_bfloat16>(&yv[x][c * 8]);
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < ROWS * 8 / NT; ++it) {
          const int idx = tid + it * NT, row = idx >> 3, c = idx & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(sPR + sw128_chunk(row, c));
          const int t_row = (n0 + g * G) * CT + row;
          stg16(static_cast<__nv_bfloat16*>(p.y) + (size_t)b * p.y_sb + (size_t)h * p.y_sh + (size_t)t_row * p.y_st +
                    c * 8,
                v);
        }
      } else if (f_valid) {
#pragma unroll
        for (int x = 0; x < G; ++x) {
          const int t_row = (n0 + g * G + x) * CT + q_chunk_row(x, f_row);
          __nv_bfloat16* yrow = static_cast<__nv_bfloat16*>(p.y) + (size_t)b * p.y_sb + (size_t)h * p.y_sh +
                                (size_t)t_row * p.y_st + e0;
#pragma unroll
          for (int e = 0; e < 16; ++e) yrow[e] = __float2bfloat16_rn(yv[x][e]);
        }
      }
    }
    // every thread's TMEM, table and tile reads are done before the next group's products
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (ok && seg == p.nseg - 1 && p.state_out && f_valid) {
    float* dst = p.state_out + (size_t)bh * 4096 + f_row * 64 + e0;
#pragma unroll
    for (int e = 0; e < 16; e += 4)
      *reinterpret_cast<float4*>(dst + e) = make_float4(Rr[e], Rr[e + 1], Rr[e + 2], Rr[e + 3]);
  }
  // after a timed-out wait: let this CTA's own loads in flight land (bounded) before exit
  if (!ok && tid == 0) {
    if (pending & 1) mbar_wait(&bars[0], kqph & 1u, 79);
    if (pending & 2) mbar_wait(&bars[1], (kqph >> 1) & 1u, 79);
    if (pending & 4) mbar_wait(&bars[2], vph, 79);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------
bool slot_mc_supported(const SlotParams& p) {
  return p.C == mc::CT && p.hd == 64 && p.rows == p.C && p.N % mc::G == 0;
}

// One CTA per SM (512 TMEM columns); segments of whole groups.  Pass A covers the segments
// before the last one; when those are fewer than the SMs, each is split into a_split equal
// pieces (a divisor of its group count) so that more CTAs share the state pass.
void slot_mc_plan(int64_t BH, int N, int* nseg, int* seg_len, int* a_split) {
  const int groups = N / mc::G, sms = num_sms();
  int s = (int)(sms / BH);
  if (s < 1) s = 1;
  if (s > groups) s = groups;
  const int len = (groups + s - 1) / s;
  *seg_len = len * mc::G;
  *nseg = (groups + len - 1) / len;
  int k = 1;
  if (*nseg > 1) {
    k = (int)(sms / (BH * (*nseg - 1)));
    if (k < 1) k = 1;
    if (k > len) k = len;
    while (len % k != 0) --k;
  }
  *a_split = k;
}

int slot_mc_fwd(const SlotParams& sp, int64_t B, int64_t in_sb, int64_t in_st, void* ws, cudaStream_t s) {
  const int64_t BH = B * sp.H;
  SlotTcParams p{};
  p.gamma = sp.gamma; p.log_a = sp.log_a; p.y = sp.y; p.y_sb = sp.y_sb; p.y_sh = sp.y_sh; p.y_st = sp.y_st;
  p.state_in = sp.state_in; p.state_out = sp.state_out;
  p.L = sp.L; p.H = sp.H; p.hd = sp.hd; p.N = sp.N;
  slot_mc_plan(BH, sp.N, &p.nseg, &p.seg_len, &p.a_split);
  p.Rseg = static_cast<float*>(ws);
  p.Dseg = p.Rseg + (size_t)BH * (p.nseg - 1 > 0 ? (p.nseg - 1) * p.a_split : 1) * 4096;
  p.y_vec = (aligned16(sp.y) && sp.y_sb % 8 == 0 && sp.y_sh % 8 == 0 && sp.y_st % 8 == 0) ? 1 : 0;
  const int64_t W = (int64_t)sp.H * sp.hd;
  const int64_t sb = B > 1 ? in_sb : (int64_t)sp.L * in_st;
  CUtensorMap mq, mk, mv;
  if (int e = slot_make_map(&mq, sp.q, W, sp.L, B, in_st, sb, 16)) return e;  // 16-row boxes (q_chunk_row)
  if (int e = slot_make_map(&mk, sp.k, W, sp.L, B, in_st, sb, mc::ROWS)) return e;
  if (int e = slot_make_map(&mv, sp.v, W, sp.L, B, in_st, sb, mc::ROWS)) return e;
  const bool ps = sp.log_a != nullptr;
  p.nseg_a = (p.nseg - 1) * p.a_split;  // pass A's pieces per (batch, head)
  if (p.nseg > 1) {
    const unsigned grid = (unsigned)(BH * p.nseg_a);
    if (ps) {
      cudaFuncSetAttribute(slot_mc_state_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mc::SMEM_A);
      slot_mc_state_kernel<true><<<grid, mc::NT, mc::SMEM_A, s>>>(mk, mv, p);
    } else {
      cudaFuncSetAttribute(slot_mc_state_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mc::SMEM_A);
      slot_mc_state_kernel<false><<<grid, mc::NT, mc::SMEM_A, s>>>(mk, mv, p);
    }
    if (int e = launch_status("slot_mc_state_kernel")) return e;
  }
  // after the state pass: a programmatic dependent launch (output CTAs take the SMs as state
  // CTAs leave them; the kernel waits before it reads the states)
  auto go = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mc::SMEM_B);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(BH * p.nseg));
    cfg.blockDim = dim3(mc::NT);
    cfg.dynamicSmemBytes = mc::SMEM_B;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.nseg > 1 ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, mq, mk, mv, p);
  };
  const cudaError_t le = ps ? go(slot_mc_out_kernel<true>) : go(slot_mc_out_kernel<false>);
  if (le != cudaSuccess) return fail((int)le, "slot_mc_out_kernel launch: %s", cudaGetErrorString(le));
  return launch_status("slot_mc_out_kernel");
}

}  // namespace hdc
