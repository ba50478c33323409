// Slot memory scan on tcgen05 tensor cores (bf16 activations, feature width 64), sm_100a.
//
// Math: the chunked decayed linear attention of the reference _slot_all_fused
// (hdcmamba/model.py:236-272); see slot_simt.cu for the formulas.  Layout and schedule:
//
//   * Work unit: one CTA per (batch*head, segment of consecutive chunks).  Pass A
//     (slot_tc_state_kernel) computes every segment's local state (from zero) and decay
//     product; pass B folds the states of the earlier segments into its entering state,
//     then walks its chunks producing outputs.
//   * Per chunk, TMA loads K, V and Q (C x 64 bf16, 128-byte swizzle) into shared memory;
//     phi and the reference's feature padding (ones for q/k, zeros for v beyond head_dim)
//     are applied in place.
//   * Tensor-core products (one thread issues tcgen05.mma; fp32 accumulators in TMEM):
//       S  = phi(Q_blk) phi(K)^T               per row block (causal columns only)
//       Y  = Qs_blk bf16(R) + P_blk V          Qs = bf16(phi(q) qdec_i), as the reference
//                                              rounds it (model.py:267-268)
//       U  = k~^T V                            k~ = bf16(phi(k) kdec_j); R <- gC R + U (fp32)
//     P = bf16(mask(S) * decay) is formed by the threads from S.
//   * Epilogue: y = bf16(Y), stored; or, with the fused gate epilogue,
//     combined = bf16(GroupNorm_head(y) * sigmoid(gate)) (hdcmamba/model.py:286-293)
//     written straight into the concatenated row.
//   * Two pass-B kernels: slot_tc_out_kernel (any chunk 64 / 128 / 256, P through shared
//     memory, all threads in lock step) and slot_tc_pipe_kernel (chunk 256 with the fused
//     gate and head_dim 64: warp-specialized, pipelined across chunks, P in TMEM).
// Decays: a table pw[k] = exp(k * log(gamma)) (constant gamma: the same expression the
// reference evaluates per element) or the chunk's cumulative log decay c_i (per-step).
#include "slot.cuh"
#include "slot_tc.cuh"

namespace hdc {

// ---------------------------------------------------------------------------------
// Pass A: per-segment local state Rseg = sum_m (prod_{m'>m} gC_m') U_m and Dseg = prod gC_m
// 16 warps; K and V of the next two chunks are in flight (two-stage TMA ring) while the
// current chunk is prepared and multiplied.  Warp w reads U rows (quarter w & 3) and the
// 16 columns [16 (w >> 2), +16) and keeps that part of R in registers.
// ---------------------------------------------------------------------------------
constexpr int kStateThreads = 512;

// (chunk 64 / 128: two CTAs per SM fit in shared memory, so registers are capped for it)
template <int CT, bool PERSTEP>
__global__ void __launch_bounds__(kStateThreads, CT == 256 ? 1 : 2)
    slot_tc_state_kernel(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV,
                         SlotTcParams p) {
  constexpr int NT = kStateThreads;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  // stage st: K at base + st * 2 * CT * 128, V right after it
  float* sTab = reinterpret_cast<float*>(base + 4 * CT * 128);  // [CT + 4]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sTab + CT + 4);   // [0], [1] stage loads, [2] MMA
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, cgrp = warp >> 2;
  const int nseg_a = p.nseg_a;
  const int bh = blockIdx.x / nseg_a, seg = blockIdx.x - bh * nseg_a;
  const int b = bh / p.H, h = bh - b * p.H;
  const int n0 = seg * p.seg_len, n1 = min(p.N, n0 + p.seg_len);

  if (warp == 0) {
    tmem_alloc(sTmem, 64);
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
  const uint32_t tU = *sTmem;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  constexpr uint32_t idU = idesc_bf16_f32(64, 64, true, true);

  float R[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) R[e] = 0.f;
  float D = 1.f;
  uint32_t fph0 = 0, fph1 = 0, mph = 0;
  int pending = 0;  // thread 0: bit st set while stage st has a load in flight
  bool ok = true;

  auto issue = [&](int n, int st) {
    uint8_t* sK = base + st * 2 * CT * 128;
    mbar_expect_tx(&bars[st], 2 * CT * 128);
    tma_load_3d(sK, &mapK, h * p.hd, n * CT, b, &bars[st]);
    tma_load_3d(sK + CT * 128, &mapV, h * p.hd, n * CT, b, &bars[st]);
    pending |= 1 << st;
  };
  if (tid == 0) {
    if (n0 < n1) issue(n0, 0);
    if (n0 + 1 < n1) issue(n0 + 1, 1);
  }
  for (int n = n0; n < n1; ++n) {
    const int st = (n - n0) & 1;
    uint8_t* sK = base + st * 2 * CT * 128;
    uint8_t* sV = sK + CT * 128;
    if (!mbar_wait_warp(&bars[st], st ? fph1 : fph0, 11)) { ok = false; break; }
    if (st) fph1 ^= 1; else fph0 ^= 1;
    if (tid == 0) pending &= ~(1 << st);
    if (PERSTEP) {
      if (warp == 0) chunk_cumlog_warp<CT>(p.log_a + ((size_t)b * p.L + (size_t)n * CT) * p.H + h, p.H, sTab);
      __syncthreads();
    }
    // k~ = bf16(bf16(phi(k)) * kdec_j) in place; v padding
#pragma unroll 2
    for (int idx = tid; idx < CT * 8; idx += NT) {
      const int row = idx >> 3, pc = idx & 7, c0 = ((pc ^ (row & 7)) << 3);
      const float kd = PERSTEP ? fast_exp(sTab[CT - 1] - sTab[row]) : sTab[CT - 1 - row];
      uint4* pk = reinterpret_cast<uint4*>(sK + row * 128 + pc * 16);
      float f[8];
      unpack16<__nv_bfloat16>(*pk, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = ((c0 + e < p.hd) ? bf16_round(phi_fast(f[e])) : 1.f) * kd;
      *pk = pack16<__nv_bfloat16>(f);
    }
    if (p.hd < 64) prep_tile<NT>(sV, CT, p.hd, false, 0.f);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < CT / 16; ++kk)
        umma_bf16(tU, sdesc_sw128(smem_u32(sK) + kk * 2048, 0, 1024), sdesc_sw128(smem_u32(sV) + kk * 2048, 0, 1024),
                  idU, kk > 0 ? 1u : 0u);
      umma_commit(&bars[2]);
    }
    if (!mbar_wait_warp(&bars[2], mph, 12)) { ok = false; break; }
    mph ^= 1;
    tc_fence_after();
    if (tid == 0 && n + 2 < n1) issue(n + 2, st);  // this stage's product is done
    const float gC = PERSTEP ? fast_exp(sTab[CT]) : sTab[CT];
    float u[16];
    tmem_ld16(tU + lane_base + cgrp * 16, u);
#pragma unroll
    for (int e = 0; e < 16; ++e) R[e] = R[e] * gC + u[e];
    D *= gC;
    // every thread's TMEM read (and, per-step, table read) is done before the next
    // chunk's product or table
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (ok && lane < 16) {
    const int f = quarter * 16 + lane;
    float* dst = p.Rseg + ((size_t)bh * p.nseg + seg) * 4096 + f * 64 + cgrp * 16;
#pragma unroll
    for (int e = 0; e < 16; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(R[e], R[e + 1], R[e + 2], R[e + 3]);
  }
  if (ok && tid == 0) p.Dseg[(size_t)bh * p.nseg + seg] = D;
  // after a timed-out wait: let this CTA's own loads in flight land (bounded) before exit
  if (!ok && tid == 0) {
    if (pending & 1) mbar_wait(&bars[0], fph0, 13);
    if (pending & 2) mbar_wait(&bars[1], fph1, 13);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tU, 64);
}

// ---------------------------------------------------------------------------------
// Pass A for chunk 256, warp-specialized (slot_tc_state_pipe_kernel): 16 compute warps
// form k~ = bf16(bf16(phi(k)) kdec_j) in place and fold R <- gC R + U in registers; one
// issue warp keeps three chunks of K and V in flight (TMA ring) and issues U = k~^T V
// into one of two TMEM buffers, so the next chunk's k~ overlaps the current product.
// Barrier phases follow from the chunk index (stage st = i % 3 completes once per 3
// chunks, U buffer i & 1 once per 2), and every wait is bounded.
// ---------------------------------------------------------------------------------
namespace spipe {
constexpr int CT = 256, NS = 3, NCW = 16, NTC = NCW * 32, NT = NTC + 32;
constexpr int TILE = CT * 128, TABN = CT + 4;
// mbarriers: TMA stage full [NS], k~ ready [NS] (per compute warp), per-step table ready
// [NS] (warp 0), U product done [2], U read [2] (per compute warp)
enum { B_FULL = 0, B_PREP = NS, B_TAB = 2 * NS, B_UFULL = 3 * NS, B_UFREE = 3 * NS + 2, NBAR = 3 * NS + 4 };
constexpr size_t SMEM = 1024 + NS * 2 * TILE + NS * TABN * 4 + NBAR * 8 + 16;
}  // namespace spipe

template <bool PERSTEP>
__global__ void __launch_bounds__(spipe::NT, 1)
    slot_tc_state_pipe_kernel(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV,
                              SlotTcParams p) {
  using namespace spipe;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  float* sTab = reinterpret_cast<float*>(base + NS * 2 * TILE);  // [NS][TABN] (constant decay: [0])
  uint64_t* bars = reinterpret_cast<uint64_t*>(sTab + NS * TABN);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + NBAR);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, cgrp = warp >> 2;
  // the output kernel (launched as this grid's programmatic dependent) may start its
  // CTAs as this grid's CTAs exit; it waits for this grid before it reads the states
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int nseg_a = p.nseg_a;
  const int bh = blockIdx.x / nseg_a, seg = blockIdx.x - bh * nseg_a;
  const int b = bh / p.H, h = bh - b * p.H;
  const int n0 = seg * p.seg_len, n1 = min(p.N, n0 + p.seg_len);
  auto sK = [&](int st) { return base + st * 2 * TILE; };
  auto sV = [&](int st) { return base + st * 2 * TILE + TILE; };
  auto tab = [&](int st) { return sTab + (PERSTEP ? st * TABN : 0); };

  if (warp == 0) {
    tmem_alloc(sTmem, 128);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i)
      mbar_init(&bars[i], ((i >= B_PREP && i < B_PREP + NS) || i >= B_UFREE) ? NCW : 1);
    fence_mbar_init();
  }
  if (!PERSTEP) {
    const float lg = logf(__bfloat162float(static_cast<const __nv_bfloat16*>(p.gamma)[h]));
    for (int k = tid; k <= CT; k += NT) sTab[k] = expf((float)k * lg);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tU = *sTmem;
  bool ok = true;

  if (warp == NCW) {
    // ------------------------------------------------------------ issue warp
    if (lane == 0 && n0 < n1) {
      tma_prefetch_map(&mapK);
      tma_prefetch_map(&mapV);
      auto load = [&](int n) {
        const int st = (n - n0) % NS;
        mbar_expect_tx(&bars[B_FULL + st], 2 * TILE);
        tma_load_3d(sK(st), &mapK, h * p.hd, n * CT, b, &bars[B_FULL + st]);
        tma_load_3d(sV(st), &mapV, h * p.hd, n * CT, b, &bars[B_FULL + st]);
      };
      for (int n = n0; n < min(n1, n0 + NS); ++n) load(n);
      constexpr uint32_t idU = idesc_bf16_f32(64, 64, true, true);
      for (int n = n0; n < n1; ++n) {
        const int i = n - n0, st = i % NS, ub = i & 1;
        if (!mbar_wait(&bars[B_PREP + st], (uint32_t)((i / NS) & 1), 71)) break;
        if (i >= 2 && !mbar_wait(&bars[B_UFREE + ub], (uint32_t)(((i >> 1) - 1) & 1), 72)) break;
        tc_fence_after();
        const uint64_t dK = sdesc_sw128(smem_u32(sK(st)), 0, 1024), dV = sdesc_sw128(smem_u32(sV(st)), 0, 1024);
#pragma unroll
        for (int kk = 0; kk < CT / 16; ++kk)
          umma_bf16(tU + ub * 64, dK + (uint64_t)((kk * 2048) >> 4), dV + (uint64_t)((kk * 2048) >> 4), idU,
                    kk > 0 ? 1u : 0u);
        umma_commit(&bars[B_UFULL + ub]);
        if (n + NS < n1) {  // this stage's product is done: refill it
          if (!mbar_wait(&bars[B_UFULL + ub], (uint32_t)((i >> 1) & 1), 73)) break;
          load(n + NS);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute warps
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float R[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) R[e] = 0.f;
    float D = 1.f, g_even = 1.f, g_odd = 1.f;  // gC of the chunks whose U is pending
    auto warp_arrive = [&](int which) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[which]);
    };
    auto prep = [&](int n) {
      const int i = n - n0, st = i % NS;
      const uint32_t ph = (uint32_t)((i / NS) & 1);
      if (!mbar_wait_warp(&bars[B_FULL + st], ph, 74)) return false;
      const float* T = tab(st);
      if (PERSTEP) {
        if (warp == 0) {
          chunk_cumlog_warp<CT>(p.log_a + ((size_t)b * p.L + (size_t)n * CT) * p.H + h, p.H, tab(st));
          warp_arrive(B_TAB + st);
        }
        if (!mbar_wait_warp(&bars[B_TAB + st], ph, 75)) return false;
      }
      const float gC = PERSTEP ? fast_exp(T[CT]) : T[CT];
      if (i & 1) g_odd = gC; else g_even = gC;
      // k~ = bf16(bf16(phi(k)) * kdec_j) in place (feature padding: k = 1)
      constexpr int IT = CT * 8 / NTC;
      uint8_t* K_ = sK(st);
      uint4 kv[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) kv[it] = reinterpret_cast<const uint4*>(K_)[tid + it * NTC];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = tid + it * NTC, row = idx >> 3, pc = idx & 7, c0 = ((pc ^ (row & 7)) << 3);
        const float kd = PERSTEP ? fast_exp(T[CT - 1] - T[row]) : T[CT - 1 - row];
        if (c0 + 8 <= p.hd) {  // packed: phi in bf16 pairs, then the fp32 product, rounded
          const uint64_t kd2 = f2_make(kd, kd);
          uint32_t* w = reinterpret_cast<uint32_t*>(&kv[it]);
#pragma unroll
          for (int i = 0; i < 4; ++i) w[i] = f2_to_bf2(f2_mul(bf2_to_f2(phi_bf2(w[i])), kd2));
          reinterpret_cast<uint4*>(K_)[idx] = kv[it];
        } else {
          float f[8];
          unpack16<__nv_bfloat16>(kv[it], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = ((c0 + e < p.hd) ? bf16_round(phi_fast(f[e])) : 1.f) * kd;
          reinterpret_cast<uint4*>(K_)[idx] = pack16<__nv_bfloat16>(f);
        }
      }
      if (p.hd < 64) prep_tile<NTC>(sV(st), CT, p.hd, false, 0.f);
      fence_proxy_async_smem();
      warp_arrive(B_PREP + st);
      return true;
    };
    if (n0 < n1) ok = prep(n0);
    for (int n = n0; n < n1 && ok; ++n) {
      const int i = n - n0, ub = i & 1;
      if (n + 1 < n1 && !prep(n + 1)) { ok = false; break; }
      if (!mbar_wait_warp(&bars[B_UFULL + ub], (uint32_t)((i >> 1) & 1), 76)) { ok = false; break; }
      tc_fence_after();
      float u[16];
      tmem_ld16(tU + ub * 64 + lane_base + cgrp * 16, u);
      tc_fence_before();
      warp_arrive(B_UFREE + ub);
      const float gC = ub ? g_odd : g_even;
#pragma unroll
      for (int e = 0; e < 16; ++e) R[e] = R[e] * gC + u[e];
      D *= gC;
    }
    if (ok && lane < 16) {
      const int f = quarter * 16 + lane;
      float* dst = p.Rseg + ((size_t)bh * p.nseg + seg) * 4096 + f * 64 + cgrp * 16;
#pragma unroll
      for (int e = 0; e < 16; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(R[e], R[e + 1], R[e + 2], R[e + 3]);
    }
    if (ok && tid == 0) p.Dseg[(size_t)bh * p.nseg + seg] = D;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tU, 128);
}

template <int CT, bool PS>
static int launch_state(const CUtensorMap& mk, const CUtensorMap& mv, const SlotTcParams& p, unsigned grid,
                        cudaStream_t s);

// ---------------------------------------------------------------------------------
// Pass B: outputs.  NWG warpgroups (NWG*128 threads); all of them cover every TMEM lane
// (row) and split the columns.  Both row blocks of a chunk go through the tensor cores
// together, so a chunk takes two round trips:
//   1. S_rb = phi(Q_rb) phi(K[0:ncol_rb])^T for every row block rb (causal columns only);
//   2. Y_rb = Qs_rb bf16(R) + P_rb V and the state update U = k~^T V (k~ and Qs are
//      formed in place between the two rounds).
// With 128-row blocks Y reuses the S columns of its block once P is read out.
// The fp32 state R stays in registers (R <- gC R + U after round 2); while round 1 runs
// the threads fetch the gate; the next chunk's loads start as soon as round 2 completes.
// ---------------------------------------------------------------------------------
template <int CT>
struct OutCfg {
  static constexpr int RB = CT < 128 ? CT : 128;        // rows per block (MMA M)
  static constexpr int NRB = CT / RB;                    // row blocks per chunk
  static constexpr int NWG = CT == 64 ? 2 : 4;           // warpgroups
  static constexpr int NT = NWG * 128;
  static constexpr int EPW = 64 / NWG;                   // accumulator columns per warpgroup
  static constexpr int AG = EPW < 16 ? EPW : 16;         // accumulator columns per TMEM access
  static constexpr int PW = NWG == 8 ? 16 : 32;          // columns of one S / P piece
  static constexpr int SRED = 2 * NWG;                   // GroupNorm partials per row
  static constexpr int MINB = CT == 64 ? 2 : 1;          // resident CTAs per SM
  static constexpr int NST = CT == 64 ? 2 : 1;           // K / V / Q stages
  static constexpr bool INPLACE = RB == 128;             // Yi / Yx inside the S columns
  static constexpr int ncol(int rb) { return (rb + 1) * RB; }      // S columns of block rb
  static constexpr int scol(int rb) { return rb == 0 ? 0 : ncol(0); }
  static constexpr int SCOLS = NRB == 1 ? ncol(0) : ncol(0) + ncol(1);
  static constexpr int yi(int rb) { return INPLACE ? scol(rb) : SCOLS; }  // Y (64 columns)
  static constexpr int RCOL = INPLACE ? SCOLS : SCOLS + 64;       // U = k~^T V (64 columns)
  static constexpr int TMEM_COLS = RCOL + 64 <= 256 ? 256 : 512;
  static constexpr int pbase(int rb) { return rb == 0 ? 0 : RB * ncol(0) * 2; }  // bytes into sP
  static constexpr int PBYTES = NRB == 1 ? RB * ncol(0) * 2 : RB * (ncol(0) + ncol(1)) * 2;
  static constexpr int NCHUNK = SCOLS / PW;              // PW-column pieces of S / P
  static constexpr int CPW = NCHUNK / NWG;               // pieces per warpgroup
  static_assert(CPW * NWG == NCHUNK, "S pieces must split evenly over the warpgroups");
};

template <int CT, bool PERSTEP, bool GATE>
__global__ void __launch_bounds__(OutCfg<CT>::NT, OutCfg<CT>::MINB)
    slot_tc_out_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                       const __grid_constant__ CUtensorMap mapV, SlotTcParams p) {
  using Cfg = OutCfg<CT>;
  constexpr int NT = Cfg::NT, RB = Cfg::RB, NRB = Cfg::NRB, NWG = Cfg::NWG, EPW = Cfg::EPW;
  constexpr int AG = Cfg::AG, PW = Cfg::PW, SRED = Cfg::SRED;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  // [NST] stages of K | V | Q (chunk 64: two, so the next chunk's loads fly during this one);
  // K holds phi(K), then k~ = bf16(phi(K) * kdec) in place
  constexpr int NST = Cfg::NST;
  uint8_t* const stage0 = base;
  uint8_t* sP = base + NST * 3 * CT * 128;  // per row block: [ncol/64 atoms][RB rows][128 B]
  uint8_t* sR = sP + Cfg::PBYTES;           // [64 rows][128 B], MN-major bf16 R
  float* sTab = reinterpret_cast<float*>(sR + 64 * 128);  // [CT + 4]
  float* sGn = sTab + CT + 4;                              // [128] gn weight | bias of this head
  float* sRed = sGn + 128;                                 // [CT][SRED] GroupNorm partial sums
  // mbarriers: [0] K + V loads of stage 0, [1] S products, [2] P.V / Yx / state products,
  // [3] Q load of stage 0, [4] K + V and [5] Q of stage 1.  Each commit follows a CTA
  // barrier, so no thread can fall two phases behind on a barrier (which would alias the
  // parity).
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRed + CT * SRED);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + 6);
  auto kv_bar = [&](int st) { return &bars[st ? 4 : 0]; };
  auto q_bar = [&](int st) { return &bars[st ? 5 : 3]; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, wg = warp >> 2;
  const int bh = blockIdx.x / p.nseg, seg = blockIdx.x - bh * p.nseg;
  const int b = bh / p.H, h = bh - b * p.H;
  const int n0 = seg * p.seg_len, n1 = min(p.N, n0 + p.seg_len);
  // accumulator row (within a row block) held by this thread (M=64: lanes 0-15 of a quarter)
  const int my_row = (RB == 128) ? quarter * 32 + lane : (lane < 16 ? quarter * 16 + lane : -1);
  const int row_lo = (RB == 128) ? quarter * 32 : quarter * 16;   // rows of this warp
  const int row_hi = row_lo + (RB == 128 ? 31 : 15);
  const bool f_valid = lane < 16;  // holds row f_row of the M=64 state R
  const int f_row = quarter * 16 + lane;
  const int e0 = wg * EPW;         // this thread's accumulator columns [e0, e0 + EPW)

  if (warp == 0) {
    tmem_alloc(sTmem, Cfg::TMEM_COLS);
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
  if (GATE) {
    for (int d = tid; d < 64; d += NT) {
      const bool in = d < p.hd;
      sGn[d] = in ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.gn_w)[h * p.hd + d]) : 0.f;
      sGn[64 + d] = in ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.gn_b)[h * p.hd + d]) : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  const uint32_t tL = tmem + lane_base;    // this warp's TMEM lanes, column 0
  const uint32_t tR = tL + Cfg::RCOL;

  // entering state: state_in, then earlier sequence parts, then the earlier segments'
  // local states, folded -> registers (fp32 R: lanes < 16 hold row f_row, columns
  // [e0, e0 + EPW)) + sR (bf16); earlier parts from other GPUs were waited for by
  // slot_wait_kernel before this launch
  float Rr[EPW];
#pragma unroll
  for (int pc = 0; pc < EPW / AG; ++pc) {
    float* Rp = Rr + pc * AG;
#pragma unroll
    for (int e = 0; e < AG; ++e) Rp[e] = 0.f;
    const int c0 = e0 + pc * AG;
    if (f_valid) {
      if (p.state_in) {
        const float* src = p.state_in + (size_t)bh * 4096 + f_row * 64 + c0;
#pragma unroll
        for (int e = 0; e < AG; ++e) Rp[e] = src[e];
      }
      // (unrolled so that the loads of several parts are in flight together)
#pragma unroll 4
      for (int s = 0; s < p.nprev; ++s) {
        const float Ds = p.prev_D[(size_t)s * p.prev_stride + bh];
        const float4* src = reinterpret_cast<const float4*>(p.prev_R + (size_t)s * p.prev_stride +
                                                            (size_t)bh * 4096 + f_row * 64 + c0);
#pragma unroll
        for (int e = 0; e < AG / 4; ++e) {
          const float4 v = src[e];
          Rp[4 * e] = Ds * Rp[4 * e] + v.x;
          Rp[4 * e + 1] = Ds * Rp[4 * e + 1] + v.y;
          Rp[4 * e + 2] = Ds * Rp[4 * e + 2] + v.z;
          Rp[4 * e + 3] = Ds * Rp[4 * e + 3] + v.w;
        }
      }
#pragma unroll 4
      for (int s = 0; s < seg; ++s) {
        const float Ds = p.Dseg[(size_t)bh * p.nseg + s];
        const float4* src = reinterpret_cast<const float4*>(p.Rseg + ((size_t)bh * p.nseg + s) * 4096 + f_row * 64 + c0);
#pragma unroll
        for (int e = 0; e < AG / 4; ++e) {
          const float4 v = src[e];
          Rp[4 * e] = Ds * Rp[4 * e] + v.x;
          Rp[4 * e + 1] = Ds * Rp[4 * e + 1] + v.y;
          Rp[4 * e + 2] = Ds * Rp[4 * e + 2] + v.z;
          Rp[4 * e + 3] = Ds * Rp[4 * e + 3] + v.w;
        }
      }
#pragma unroll
      for (int c = 0; c < AG / 8; ++c)
        *reinterpret_cast<uint4*>(sR + sw128_chunk(f_row, (c0 >> 3) + c)) = pack16<__nv_bfloat16>(&Rp[c * 8]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  constexpr uint32_t idPV = idesc_bf16_f32(RB, 64, false, true);
  constexpr uint32_t idU = idesc_bf16_f32(64, 64, true, true);

  uint32_t kph = 0, qph = 0, sph = 0, pph = 0;  // kph / qph: parity bit per stage
  int pending = 0;  // thread 0: bit st set while stage st has loads in flight
  bool ok = true;
  auto issue = [&](int n, int st) {
    uint8_t* k_ = stage0 + st * 3 * CT * 128;
    mbar_expect_tx(kv_bar(st), 2 * CT * 128);
    tma_load_3d(k_, &mapK, h * p.hd, n * CT, b, kv_bar(st));
    tma_load_3d(k_ + CT * 128, &mapV, h * p.hd, n * CT, b, kv_bar(st));
    mbar_expect_tx(q_bar(st), CT * 128);
    tma_load_3d(k_ + 2 * CT * 128, &mapQ, h * p.hd, n * CT, b, q_bar(st));
    pending |= 1 << st;
  };
  if (tid == 0) {
    for (int i = 0; i < NST && n0 + i < n1; ++i) issue(n0 + i, i);
  }

  for (int n = n0; n < n1 && ok; ++n) {
    const int st = NST == 2 ? ((n - n0) & 1) : 0;
    uint8_t* const sK = stage0 + st * 3 * CT * 128;
    uint8_t* const sV = sK + CT * 128;
    uint8_t* const sQ = sV + CT * 128;
    if (!mbar_wait_warp(kv_bar(st), (kph >> st) & 1u, 21) || !mbar_wait_warp(q_bar(st), (qph >> st) & 1u, 22)) {
      ok = false;
      break;
    }
    kph ^= 1u << st;
    qph ^= 1u << st;
    if (tid == 0) pending &= ~(1 << st);
    if (PERSTEP) {
      if (warp == 0) chunk_cumlog_warp<CT>(p.log_a + ((size_t)b * p.L + (size_t)n * CT) * p.H + h, p.H, sTab);
      __syncthreads();
    }
    // phi in place (feature padding: ones for q / k, zeros for v)
    prep_tile_u<NT, CT, true>(sK, p.hd, 1.f);
    prep_tile_u<NT, CT, true>(sQ, p.hd, 1.f);
    if (p.hd < 64) prep_tile_u<NT, CT, false>(sV, p.hd, 0.f);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- round 1: S of every row block
    if (tid == 0) {
#pragma unroll
      for (int rb = 0; rb < NRB; ++rb) {
        const uint32_t aq = smem_u32(sQ) + rb * RB * 128;
        const uint32_t idS = idesc_bf16_f32(RB, Cfg::ncol(rb), false, false);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tmem + Cfg::scol(rb), sdesc_sw128(aq + k * 32, 16, 1024),
                    sdesc_sw128(smem_u32(sK) + k * 32, 16, 1024), idS, k > 0 ? 1u : 0u);
      }
      umma_commit(&bars[1]);
    }
    // meanwhile: this thread's gate values
    uint4 graw[NRB][EPW / 8];
    if (GATE) {
#pragma unroll
      for (int rb = 0; rb < NRB; ++rb) {
        const int t_row = n * CT + rb * RB + (my_row >= 0 ? my_row : 0);
        const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(p.gate) + (size_t)b * p.g_sb +
                                  (size_t)t_row * p.g_st + (size_t)h * p.hd + e0;
#pragma unroll
        for (int c = 0; c < EPW / 8; ++c)
          graw[rb][c] = ldg16_pred(gp + c * 8, my_row >= 0 && e0 + c * 8 < p.hd);
      }
    }
    if (!mbar_wait_warp(&bars[1], sph, 23)) { ok = false; break; }
    sph ^= 1;
    tc_fence_after();
    // k~ = bf16(phi(k) * kdec_j) and Qs = bf16(phi(q) * qdec_i) in place (the S products no
    // longer read sK / sQ; the reference rounds the q-decayed queries before the state
    // product, hdcmamba/model.py:267-268)
    for (int idx = tid; idx < CT * 8; idx += NT) {
      const int row = idx >> 3;
      const float kd = PERSTEP ? fast_exp(sTab[CT - 1] - sTab[row]) : sTab[CT - 1 - row];
      const float qd = PERSTEP ? fast_exp(sTab[row]) : sTab[row];
      float f[8];
      unpack16<__nv_bfloat16>(reinterpret_cast<const uint4*>(sK)[idx], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= kd;
      reinterpret_cast<uint4*>(sK)[idx] = pack16<__nv_bfloat16>(f);
      unpack16<__nv_bfloat16>(reinterpret_cast<const uint4*>(sQ)[idx], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= qd;
      reinterpret_cast<uint4*>(sQ)[idx] = pack16<__nv_bfloat16>(f);
    }
    // P = bf16(mask(S) * decay): this warpgroup's 32-column pieces of S -> sP
#pragma unroll
    for (int cc = 0; cc < Cfg::CPW; ++cc) {
      const int c = wg * Cfg::CPW + cc;
      const int rb = (NRB == 2 && c * PW >= Cfg::ncol(0)) ? 1 : 0;
      const int j0 = c * PW - (rb ? Cfg::ncol(0) : 0);           // first column of the piece
      const int ib = rb * RB;                                     // first row of the block
      uint8_t* pb = sP + Cfg::pbase(rb);
      if (j0 > ib + row_hi) {  // above the diagonal for every row of this warp: zeros
        if (my_row >= 0) {
#pragma unroll
          for (int q = 0; q < PW / 8; ++q)
            *reinterpret_cast<uint4*>(pb + ((j0 + q * 8) >> 6) * (RB * 128) +
                                      sw128_chunk(my_row, ((j0 + q * 8) & 63) >> 3)) = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      float sv[PW];
      tmem_ldn<PW>(tL + Cfg::scol(rb) + j0, sv);
      if (my_row < 0) continue;
      const int i = ib + my_row;
      const bool full = j0 + PW - 1 <= ib + row_lo;  // no masking for any row of this warp
      const float ci = PERSTEP ? sTab[i] : 0.f;
#pragma unroll
      for (int q = 0; q < PW / 8; ++q) {
        float v[8];
        if (!PERSTEP && full) {
          // gamma^(i-j) = gamma^(i-j0-8q-7) * gamma^(7-e) for j = j0 + 8q + e
          const float rf = sTab[i - j0 - q * 8 - 7];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = sv[q * 8 + e] * (rf * sTab[7 - e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = j0 + q * 8 + e;
            float dm = 0.f;
            if (j <= i) dm = PERSTEP ? fast_exp(ci - sTab[j]) : sTab[i - j];
            v[e] = (j <= i) ? sv[q * 8 + e] * dm : 0.f;
          }
        }
        const int jq = j0 + q * 8;
        *reinterpret_cast<uint4*>(pb + (jq >> 6) * (RB * 128) + sw128_chunk(my_row, (jq & 63) >> 3)) =
            pack16<__nv_bfloat16>(v);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- round 2: Y = Qs bf16(R) + P V per row block; U = k~^T V
    if (tid == 0) {
#pragma unroll
      for (int rb = 0; rb < NRB; ++rb) {
        const uint32_t aq = smem_u32(sQ) + rb * RB * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tmem + Cfg::yi(rb), sdesc_sw128(aq + k * 32, 16, 1024),
                    sdesc_sw128(smem_u32(sR) + k * 2048, 0, 1024), idPV, k > 0 ? 1u : 0u);
        const uint32_t ap = smem_u32(sP + Cfg::pbase(rb));
        for (int kk = 0; kk < Cfg::ncol(rb) / 16; ++kk)
          umma_bf16(tmem + Cfg::yi(rb), sdesc_sw128(ap + ((kk * 16) >> 6) * (RB * 128) + ((kk * 16) & 63) * 2, 16, 1024),
                    sdesc_sw128(smem_u32(sV) + kk * 16 * 128, 0, 1024), idPV, 1u);
      }
#pragma unroll
      for (int kk = 0; kk < CT / 16; ++kk)  // U = k~^T V
        umma_bf16(tmem + Cfg::RCOL, sdesc_sw128(smem_u32(sK) + kk * 2048, 0, 1024),
                  sdesc_sw128(smem_u32(sV) + kk * 2048, 0, 1024), idU, kk > 0 ? 1u : 0u);
      umma_commit(&bars[2]);
    }
    if (!mbar_wait_warp(&bars[2], pph, 24)) { ok = false; break; }
    pph ^= 1;
    tc_fence_after();
    if (tid == 0 && n + NST < n1) issue(n + NST, st);  // every buffer of this chunk's stage is free
    // ---- epilogue: y = bf16(Y), plain or GroupNorm * sigmoid(gate)
    float o[NRB][EPW];
#pragma unroll
    for (int rb = 0; rb < NRB; ++rb) {
#pragma unroll
      for (int pc = 0; pc < EPW / AG; ++pc) {
        float yi[AG];
        tmem_ldn<AG>(tL + Cfg::yi(rb) + e0 + pc * AG, yi);
#pragma unroll
        for (int e = 0; e < AG; ++e) o[rb][pc * AG + e] = bf16_round(yi[e]);  // y_slot is bf16
      }
    }
    if (GATE) {
      float mean[NRB];
#pragma unroll
      for (int rb = 0; rb < NRB; ++rb) {
        float sum = 0.f;
#pragma unroll
        for (int e = 0; e < EPW; ++e) sum += (e0 + e < p.hd) ? o[rb][e] : 0.f;
        if (my_row >= 0) sRed[(rb * RB + my_row) * SRED + wg] = sum;
      }
      named_bar_sync(1 + quarter, NWG * 32);  // the warps holding these rows
#pragma unroll
      for (int rb = 0; rb < NRB; ++rb) {
        mean[rb] = 0.f;
        if (my_row >= 0) {
#pragma unroll
          for (int w = 0; w < NWG; ++w) mean[rb] += sRed[(rb * RB + my_row) * SRED + w];
          mean[rb] *= fast_rcp((float)p.hd);
        }
        float sq = 0.f;
#pragma unroll
        for (int e = 0; e < EPW; ++e) {
          const float d = o[rb][e] - mean[rb];
          sq += (e0 + e < p.hd) ? d * d : 0.f;
        }
        if (my_row >= 0) sRed[(rb * RB + my_row) * SRED + NWG + wg] = sq;
      }
      named_bar_sync(1 + quarter, NWG * 32);
      if (my_row >= 0) {
#pragma unroll
        for (int rb = 0; rb < NRB; ++rb) {
          float ssq = 0.f;
#pragma unroll
          for (int w = 0; w < NWG; ++w) ssq += sRed[(rb * RB + my_row) * SRED + NWG + w];
          // the reference's padded lanes (block width 64) add (64 - hd) * mean^2
          const float var = (ssq + (float)(64 - p.hd) * mean[rb] * mean[rb]) / (float)p.hd;
          const float inv = rsqrtf(var + 1e-5f);
          const int t_row = n * CT + rb * RB + my_row;
          __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.y) + (size_t)b * p.y_sb + (size_t)h * p.y_sh +
                              (size_t)t_row * p.y_st + e0;
#pragma unroll
          for (int c = 0; c < EPW / 8; ++c) {
            if (e0 + c * 8 >= p.hd) continue;
            float g[8], r[8];
            unpack16<__nv_bfloat16>(graw[rb][c], g);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int d = e0 + c * 8 + e;
              const float ygn = ((o[rb][c * 8 + e] - mean[rb]) * inv) * sGn[d] + sGn[64 + d];
              r[e] = ygn * fast_sigmoid(g[e]);
            }
            stg16(op + c * 8, pack16<__nv_bfloat16>(r));
          }
        }
      }
    } else if (my_row >= 0) {
#pragma unroll
      for (int rb = 0; rb < NRB; ++rb) {
        const int t_row = n * CT + rb * RB + my_row;
        __nv_bfloat16* yrow = static_cast<__nv_bfloat16*>(p.y) + (size_t)b * p.y_sb + (size_t)h * p.y_sh +
                              (size_t)t_row * p.y_st + e0;
        if (p.y_vec) {
#pragma unroll
          for (int c = 0; c < EPW / 8; ++c)
            if (e0 + c * 8 < p.hd) stg16(yrow + c * 8, pack16<__nv_bfloat16>(&o[rb][c * 8]));
        } else {
#pragma unroll
          for (int e = 0; e < EPW; ++e)
            if (e0 + e < p.hd) yrow[e] = __float2bfloat16_rn(o[rb][e]);
        }
      }
    }
    // R <- gC * R + U (fp32) -> sR (bf16) for the next chunk's Yx
    {
      const float gC = PERSTEP ? fast_exp(sTab[CT]) : sTab[CT];
#pragma unroll
      for (int pc = 0; pc < EPW / AG; ++pc) {
        float u[AG];
        tmem_ldn<AG>(tR + e0 + pc * AG, u);
        float* Rp = Rr + pc * AG;
#pragma unroll
        for (int e = 0; e < AG; ++e) Rp[e] = fmaf(Rp[e], gC, u[e]);
        if (f_valid) {
#pragma unroll
          for (int c = 0; c < AG / 8; ++c)
            *reinterpret_cast<uint4*>(sR + sw128_chunk(f_row, ((e0 + pc * AG) >> 3) + c)) =
                pack16<__nv_bfloat16>(&Rp[c * 8]);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  // after a timed-out wait: let this CTA's own loads in flight land (bounded) before exit
  if (!ok && tid == 0) {
    for (int st = 0; st < NST; ++st) {
      if (pending & (1 << st)) {
        mbar_wait(kv_bar(st), (kph >> st) & 1u, 26);
        mbar_wait(q_bar(st), (qph >> st) & 1u, 27);
      }
    }
  }
  if (ok && seg == p.nseg - 1 && p.state_out) {
#pragma unroll
    for (int pc = 0; pc < EPW / AG; ++pc) {
      const float* r = Rr + pc * AG;
      if (f_valid) {
        float* dst = p.state_out + (size_t)bh * 4096 + f_row * 64 + e0 + pc * AG;
#pragma unroll
        for (int e = 0; e < AG; e += 4)
          *reinterpret_cast<float4*>(dst + e) = make_float4(r[e], r[e + 1], r[e + 2], r[e + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

// ---------------------------------------------------------------------------------
// Pass B for chunk 256, warp-specialized and software-pipelined across chunks
// (slot_tc_pipe_kernel).  16 compute warps (512 threads) and one issue warp (warp 16,
// one thread): TMA loads and stores, tcgen05.mma, commits.  Shared memory: phi(K) / phi(Q)
// of two chunks (stages alternate), V of one chunk, the gate tile of one chunk (the gated
// outputs are written over it and leave by one TMA store), R as bf16.  P lives in TMEM.
// Per chunk n (stage cur, next chunk's stage nxt), compute warps:
//   wait S(n)                 S_rb = phi(Q_rb) phi(K)^T
//   k~ = bf16(phi(k) kdec_j), Qs = bf16(phi(q) qdec_i) in place (the reference rounds the
//   q-decayed queries before the state product, hdcmamba/model.py:267-268);
//   P = bf16(mask(S) decay) into TMEM                                      -> arrive P
//   phi of chunk n+1's Q and K                      || issue warp: Y_rb = Qs_rb bf16(R) + P_rb V,
//                                                                  U = k~^T V
//   wait Y; y = bf16(Y), GroupNorm partial sums; R <- gC R + U -> bf16 R  -> arrive ready
//   GroupNorm * sigmoid(gate) over the gate tile                        -> arrive out
//                                                   || issue warp: S(n+1), TMA store of
//                                                      chunk n's outputs, gate of n+1
// TMEM (512 columns): S of row block 0 in [0,128), of row block 1 in [128,384), cut in
// 16-column pieces.  A row-block-0 piece keeps its P (8 packed columns) in its own first
// half; row block 1's P goes to [384,512).  Y and U are written only by the second round of
// products, which starts after every warp has read its S pieces, so they take row block
// 1's S columns: Y_rb in [128 + 64 rb, +64), U in [256,320).
// Every wait is bounded; compute warps synchronise with each other through an mbarrier
// (bounded wait), never through bar.sync inside the loop.
// ---------------------------------------------------------------------------------
namespace pipe {
constexpr int CT = 256, RB = 128, NWG = 4, NCW = NWG * 4, NTC = NCW * 32, NT = NTC + 32, EPW = 16, PW = 16;
constexpr int NPIECE = 3 * RB / PW;  // 24 pieces of S (8 of row block 0, 16 of row block 1)
constexpr int CPW = NPIECE / NWG;    // per warpgroup
constexpr int YCOL = RB, UCOL = 2 * RB, P1COL = 3 * RB;
constexpr int TILE = CT * 128;       // one [CT x 64] bf16 tile
constexpr int TABN = CT + 4;
// mbarriers
enum { B_L0, B_L1, B_V, B_G, B_S, B_Y, B_READY, B_P, B_KQ, B_OUT, B_SYNC, NBAR };
constexpr size_t SMEM = 1024 + 6 * TILE + 64 * 128 + 2 * TABN * 4 + 128 * 4 + 2 * CT * NWG * 8 + NBAR * 8 + 16;
// Chunk row held by Q tile row r (and by TMEM lane r of row block 0's accumulators): row
// block 0 arrives in 32-row blocks in reverse order, so every lane quarter holds one block of
// row block 0 and one of row block 1 whose causal widths add up to the same total (P work
// balanced over the warps).  Row block 1 is in order.
__host__ __device__ constexpr int q_row(int r) { return r < RB ? (RB - 32) - (r & ~31) + (r & 31) : r; }
// TMEM column of the packed P of piece c (row block 0: in place; row block 1: [384,512))
__device__ __forceinline__ uint32_t pcol(int c) {
  return c < RB / PW ? (uint32_t)(c * PW) : (uint32_t)(P1COL + (c - RB / PW) * (PW / 2));
}
}  // namespace pipe

// gate / output tensor maps travel with the parameters
struct SlotPipeMaps {
  CUtensorMap gate, out;
};

// LATE: the earlier sequence parts' states arrive from other GPUs behind wait flags (a
// separate instantiation, so the single-GPU kernel keeps its register allocation)
template <bool PERSTEP, bool LATE>
__global__ void __launch_bounds__(pipe::NT, 1)
    slot_tc_pipe_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                        const __grid_constant__ CUtensorMap mapV, const __grid_constant__ SlotPipeMaps mg,
                        SlotTcParams p) {
  using namespace pipe;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  // [0,4): K0 Q0 K1 Q1, [4] V, [5] gate / outputs
  uint8_t* sV = base + 4 * TILE;
  uint8_t* sG = base + 5 * TILE;
  uint8_t* sR = base + 6 * TILE;                           // [64 rows][128 B], MN-major bf16 R
  float* sTab = reinterpret_cast<float*>(sR + 64 * 128);  // [2][TABN] (per-step: one per stage)
  float* sGn = sTab + 2 * TABN;                            // [128] gn weight | bias of this head
  float2* sRed = reinterpret_cast<float2*>(sGn + 128);     // [2][NWG][CT] GroupNorm (sum, sum of squares)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRed + 2 * CT * NWG);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + NBAR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, wg = warp >> 2;
  const bool issuer = warp == NCW;
  const int bh = blockIdx.x / p.nseg, seg = blockIdx.x - bh * p.nseg;
  const int b = bh / p.H, h = bh - b * p.H;
  const int n0 = seg * p.seg_len, n1 = min(p.N, n0 + p.seg_len);
  const int my_row = quarter * 32 + lane;  // accumulator row within a row block
  const int row_lo = quarter * 32, row_hi = row_lo + 31;
  const bool f_valid = lane < 16;          // holds row f_row of the M=64 products (U)
  const int f_row = quarter * 16 + lane;
  const int e0 = wg * EPW;                 // this thread's accumulator columns [e0, e0 + 16)

  auto sK = [&](int st) { return base + (2 * st) * TILE; };
  auto sQ = [&](int st) { return base + (2 * st + 1) * TILE; };
  auto tab = [&](int st) { return sTab + (PERSTEP ? st * TABN : 0); };

  if (warp == 0) {
    tmem_alloc(sTmem, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i)
      mbar_init(&bars[i], (i == B_READY || i == B_P || i == B_KQ || i == B_OUT || i == B_SYNC) ? NCW : 1);
    fence_mbar_init();
  }
  if (!PERSTEP) {
    const float lg = logf(__bfloat162float(static_cast<const __nv_bfloat16*>(p.gamma)[h]));
    for (int k = tid; k <= CT; k += NT) sTab[k] = expf((float)k * lg);
  }
  for (int d = tid; d < 64; d += NT) {
    sGn[d] = __bfloat162float(static_cast<const __nv_bfloat16*>(p.gn_w)[h * 64 + d]);
    sGn[64 + d] = __bfloat162float(static_cast<const __nv_bfloat16*>(p.gn_b)[h * 64 + d]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;

  if (issuer) {
    // ------------------------------------------------------------ issue warp
    if (lane == 0 && n0 < n1) {
      tma_prefetch_map(&mapQ);
      tma_prefetch_map(&mapK);
      tma_prefetch_map(&mapV);
      auto load_kq = [&](int n, int st) {
        mbar_expect_tx(&bars[B_L0 + st], 2 * TILE);
        tma_load_3d(sK(st), &mapK, h * p.hd, n * CT, b, &bars[B_L0 + st]);
        // Q in 32-row boxes; row block 0's blocks in reverse order (q_row)
#pragma unroll
        for (int j = 0; j < CT / 32; ++j)
          tma_load_3d(sQ(st) + j * 32 * 128, &mapQ, h * p.hd, n * CT + q_row(j * 32), b, &bars[B_L0 + st]);
      };
      auto load_v = [&](int n) {
        mbar_expect_tx(&bars[B_V], TILE);
        tma_load_3d(sV, &mapV, h * p.hd, n * CT, b, &bars[B_V]);
      };
      auto load_g = [&](int n) {
        mbar_expect_tx(&bars[B_G], TILE);
        tma_load_3d(sG, &mg.gate, h * p.hd, n * CT, b, &bars[B_G]);
      };
      load_kq(n0, 0);
      load_v(n0);
      load_g(n0);
      if (n0 + 1 < n1) load_kq(n0 + 1, 1);
      constexpr uint32_t idPV = idesc_bf16_f32(RB, 64, false, true);
      constexpr uint32_t idU = idesc_bf16_f32(64, 64, true, true);
      uint32_t rph = 0, pph = 0, kqph = 0, yph = 0, oph = 0;
      for (int n = n0; n < n1; ++n) {
        const int cur = (n - n0) & 1;
        // S_rb = phi(Q_rb) phi(K[0 : 128 (rb + 1)])^T once phi(n) is in place and Y(n-1), U(n-1)
        // were read out of TMEM
        if (!mbar_wait(&bars[B_READY], rph, 51)) break;
        rph ^= 1;
        tc_fence_after();
        // descriptors of the stage's tiles; an MMA's operand is the base plus offset / 16
        const uint64_t dK = sdesc_sw128(smem_u32(sK(cur)), 16, 1024), dQ = sdesc_sw128(smem_u32(sQ(cur)), 16, 1024);
        // the two row blocks' accumulations interleaved (independent chains overlap in the
        // tensor pipe)
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
            umma_bf16(tmem + rb * RB, dQ + (uint64_t)((rb * RB * 128 + k * 32) >> 4), dK + (uint64_t)((k * 32) >> 4),
                      idesc_bf16_f32(RB, RB * (rb + 1), false, false), k > 0 ? 1u : 0u);
        umma_commit(&bars[B_S]);
        // Y_rb = P_rb V + Qs_rb bf16(R);  U = k~^T V.  The P V products go first: they need only
        // P (TMEM) and V, so they run while the compute warps form k~ and Qs in place.
        if (!mbar_wait(&bars[B_P], pph, 53)) break;
        pph ^= 1;
        if (!mbar_wait(&bars[B_V], (uint32_t)((n - n0) & 1), 54)) break;
        tc_fence_after();
        const uint64_t dR = sdesc_sw128(smem_u32(sR), 0, 1024), dV = sdesc_sw128(smem_u32(sV), 0, 1024);
        const uint64_t dKm = sdesc_sw128(smem_u32(sK(cur)), 0, 1024);
        constexpr int KPP = PW / 16;  // 16-column K steps per piece
        auto pv_step = [&](int rb, int kk) {  // K step kk of P_rb V (the first one starts Y_rb)
          const int c = rb * (RB / PW) + kk / KPP;
          umma_bf16_ts(tmem + YCOL + 64 * rb, tmem + pcol(c) + (kk % KPP) * 8, dV + (uint64_t)((kk * 16 * 128) >> 4),
                       idPV, kk > 0 ? 1u : 0u);
        };
        // two independent accumulations, interleaved: Y_1 (16 steps), Y_0 (8)
#pragma unroll
        for (int t = 0; t < 2 * RB / 16; ++t) {
          pv_step(1, t);
          if (t < RB / 16) pv_step(0, t);
        }
        if (!mbar_wait(&bars[B_KQ], kqph, 64)) break;
        kqph ^= 1;
        tc_fence_after();
        // U (16 steps) interleaved with Qs_rb bf16(R) (4 steps per row block, accumulating)
#pragma unroll
        for (int t = 0; t < CT / 16; ++t) {
          umma_bf16(tmem + UCOL, dKm + (uint64_t)((t * 2048) >> 4), dV + (uint64_t)((t * 2048) >> 4), idU,
                    t > 0 ? 1u : 0u);
          if (t < 4) {
#pragma unroll
            for (int rb = 0; rb < 2; ++rb)
              umma_bf16(tmem + YCOL + 64 * rb, dQ + (uint64_t)((rb * RB * 128 + t * 32) >> 4),
                        dR + (uint64_t)((t * 2048) >> 4), idPV, 1u);
          }
        }
        umma_commit(&bars[B_Y]);
        // every product reading stage cur and V is done: next loads
        if (!mbar_wait(&bars[B_Y], yph, 55)) break;
        yph ^= 1;
        if (n + 1 < n1) load_v(n + 1);
        if (n + 2 < n1) load_kq(n + 2, cur);
        // the gated outputs of chunk n-1 (formed during this chunk's products) out, the gate
        // tile of chunk n in
        if (n > n0) {
          if (!mbar_wait(&bars[B_OUT], oph, 52)) break;
          oph ^= 1;
          tma_store_3d(&mg.out, sG, h * p.hd, (n - 1) * CT, b);
          bulk_commit();
          bulk_wait_read0();
          load_g(n);
        }
      }
      // outputs of the last chunk
      if (mbar_wait(&bars[B_OUT], oph, 56)) {
        tma_store_3d(&mg.out, sG, h * p.hd, (n1 - 1) * CT, b);
        bulk_commit();
      }
      bulk_wait0();
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute warps
    const uint32_t tL = tmem + ((uint32_t)(quarter * 32) << 16);  // this warp's TMEM lanes
    float Rr[EPW];
#pragma unroll
    for (int e = 0; e < EPW; ++e) Rr[e] = 0.f;
    uint32_t lph0 = 0, lph1 = 0, sph = 0, yph = 0, gph = 0;
    bool ok = true;
    // one arrival per compute warp, after every lane's writes and fences
    auto warp_arrive = [&](int which) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[which]);
    };
    // phi of a stage's Q and K in place (padding: ones), per-step decay table by warp 0
    auto prep = [&](int n, int st) {
      if (!mbar_wait_warp(&bars[B_L0 + st], st ? lph1 : lph0, 57)) return false;
      if (st) lph1 ^= 1; else lph0 ^= 1;
      if (PERSTEP && warp == 0)
        chunk_cumlog_warp<CT>(p.log_a + ((size_t)b * p.L + (size_t)n * CT) * p.H + h, p.H, tab(st));
      prep_tile_u<NTC, CT, true>(sK(st), 64, 1.f);
      prep_tile_u<NTC, CT, true>(sQ(st), 64, 1.f);
      fence_proxy_async_smem();
      return true;
    };
    // y of the chunk whose GroupNorm * gate is pending, as bf16 pairs (it is stored as bf16)
    uint32_t yp[2][EPW / 2];
    // outputs of chunk m: GroupNorm(y) * sigmoid(gate) over the gate tile, with the
    // GroupNorm partials every warp left in sRed[(m - n0) & 1]
    auto gn_gate = [&](int m) -> bool {
      if (!mbar_wait_warp(&bars[B_SYNC], (uint32_t)((m - n0) & 1), 61)) return false;
      if (!mbar_wait_warp(&bars[B_G], gph, 62)) return false;
      gph ^= 1;
      const float2* red = sRed + (size_t)((m - n0) & 1) * (NWG * CT);
#pragma unroll
      for (int rb = 0; rb < 2; ++rb) {
        const int row = rb * RB + my_row;
        float S1 = 0.f, S2 = 0.f;
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
          const float2 v = red[w * CT + row];
          S1 += v.x;
          S2 += v.y;
        }
        const float mean = S1 * (1.f / 64.f);
        const float var = fmaxf(S2 - S1 * mean, 0.f) * (1.f / 64.f);
        const float inv = rsqrtf(var + 1e-5f);
        const uint64_t mean2 = f2_make(mean, mean), inv2 = f2_make(inv, inv), half2 = f2_make(0.5f, 0.5f);
#pragma unroll
        for (int c = 0; c < EPW / 8; ++c) {
          uint4* gs = reinterpret_cast<uint4*>(sG + sw128_chunk(q_row(row), (e0 >> 3) + c));
          uint4 gv = *gs;
          uint32_t* w = reinterpret_cast<uint32_t*>(&gv);
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const int d = e0 + c * 8 + e;
            // ((y - mean) * inv) * w + b, then * sigmoid(g) = * (0.5 tanh(g / 2) + 0.5)
            const float2 gw = *reinterpret_cast<const float2*>(&sGn[d]);
            const float2 gb = *reinterpret_cast<const float2*>(&sGn[64 + d]);
            const uint64_t ygn = f2_fma(f2_mul(f2_sub(bf2_to_f2(yp[rb][(c * 8 + e) / 2]), mean2), inv2),
                                        f2_make(gw.x, gw.y), f2_make(gb.x, gb.y));
            float tl, th;
            f2_split(f2_mul(bf2_to_f2(w[e / 2]), half2), tl, th);
            asm("tanh.approx.f32 %0, %0;" : "+f"(tl));
            asm("tanh.approx.f32 %0, %0;" : "+f"(th));
            w[e / 2] = f2_to_bf2(f2_mul(ygn, f2_fma(half2, f2_make(tl, th), half2)));
          }
          *gs = gv;
        }
      }
      fence_proxy_async_smem();
      warp_arrive(B_OUT);
      return true;
    };

    if (n0 < n1) {
      ok = prep(n0, 0);
      tc_fence_before();
      warp_arrive(B_READY);
    }
    // the entering state (read by the Qs R products of the first chunk, after its k~ / Qs)
    // is folded while S(n0) runs
    // state_in, then earlier sequence parts, then the earlier segments' local states (lanes
    // < 16 hold row f_row, columns [e0, e0 + 16)) -> registers + sR.  When the earlier parts
    // arrive from other GPUs (wait flags), only this segment's predecessors are folded here
    // (Rr, with the product of their decays in Dloc); the parts are waited for and folded in
    // after the first chunk's P, R = Dloc R_parts + Rr, so the wait overlaps this CTA's
    // prologue, the first loads, phi, S and P.
    // the segment states come from the state pass: when this kernel was launched as its
    // programmatic dependent, everything above (loads, phi and S of the first chunk) ran
    // while that pass was finishing; wait for it here (returns at once otherwise)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    constexpr bool late = LATE;
    float Dloc = 1.f;
    if (f_valid && late) {
#pragma unroll 4
      for (int s = 0; s < seg; ++s) {
        const float Ds = p.Dseg[(size_t)bh * p.nseg + s];
        const float4* src =
            reinterpret_cast<const float4*>(p.Rseg + ((size_t)bh * p.nseg + s) * 4096 + f_row * 64 + e0);
#pragma unroll
        for (int e = 0; e < EPW / 4; ++e) {
          const float4 v = src[e];
          Rr[4 * e] = Ds * Rr[4 * e] + v.x;
          Rr[4 * e + 1] = Ds * Rr[4 * e + 1] + v.y;
          Rr[4 * e + 2] = Ds * Rr[4 * e + 2] + v.z;
          Rr[4 * e + 3] = Ds * Rr[4 * e + 3] + v.w;
        }
        Dloc *= Ds;
      }
    }
    if (f_valid && !late) {
      if (p.state_in) {
        const float* src = p.state_in + (size_t)bh * 4096 + f_row * 64 + e0;
#pragma unroll
        for (int e = 0; e < EPW; ++e) Rr[e] = src[e];
      }
#pragma unroll 4
      for (int s = 0; s < p.nprev; ++s) {
        const float Ds = p.prev_D[(size_t)s * p.prev_stride + bh];
        const float4* src = reinterpret_cast<const float4*>(p.prev_R + (size_t)s * p.prev_stride +
                                                            (size_t)bh * 4096 + f_row * 64 + e0);
#pragma unroll
        for (int e = 0; e < EPW / 4; ++e) {
          const float4 v = src[e];
          Rr[4 * e] = Ds * Rr[4 * e] + v.x;
          Rr[4 * e + 1] = Ds * Rr[4 * e + 1] + v.y;
          Rr[4 * e + 2] = Ds * Rr[4 * e + 2] + v.z;
          Rr[4 * e + 3] = Ds * Rr[4 * e + 3] + v.w;
        }
      }
#pragma unroll 4
      for (int s = 0; s < seg; ++s) {
        const float Ds = p.Dseg[(size_t)bh * p.nseg + s];
        const float4* src =
            reinterpret_cast<const float4*>(p.Rseg + ((size_t)bh * p.nseg + s) * 4096 + f_row * 64 + e0);
#pragma unroll
        for (int e = 0; e < EPW / 4; ++e) {
          const float4 v = src[e];
          Rr[4 * e] = Ds * Rr[4 * e] + v.x;
          Rr[4 * e + 1] = Ds * Rr[4 * e + 1] + v.y;
          Rr[4 * e + 2] = Ds * Rr[4 * e + 2] + v.z;
          Rr[4 * e + 3] = Ds * Rr[4 * e + 3] + v.w;
        }
      }
#pragma unroll
      for (int c = 0; c < EPW / 8; ++c)
        *reinterpret_cast<uint4*>(sR + sw128_chunk(f_row, (e0 >> 3) + c)) = pack16<__nv_bfloat16>(&Rr[c * 8]);
    }


    // warp 0's per-step table of chunk n0 is visible to every compute warp (every compute
    // warp passes this barrier exactly once)
    if (PERSTEP) named_bar_sync(1, NTC);
    for (int n = n0; n < n1 && ok; ++n) {
      const int cur = (n - n0) & 1, nxt = cur ^ 1;
      uint8_t* K_ = sK(cur);
      uint8_t* Q_ = sQ(cur);
      const float* T = tab(cur);
      // per-step: warp 0 wrote chunk n's table (in prep(n), before its arrival at the end of
      // chunk n-1)
      if (PERSTEP && n > n0 && !mbar_wait_warp(&bars[B_SYNC], (uint32_t)((n - 1 - n0) & 1), 63)) {
        ok = false;
        break;
      }
      if (!mbar_wait_warp(&bars[B_S], sph, 58)) { ok = false; break; }
      sph ^= 1;
      tc_fence_after();
      // P = bf16(mask(S) decay) of this warpgroup's pieces -> TMEM (packed pairs)
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int c = cc * NWG + wg;      // pieces interleaved over the warpgroups
        const int rb = c * PW >= RB ? 1 : 0;
        const int j0 = c * PW - rb * RB;  // chunk position of the piece's first column
        const int rlo = q_row(rb * RB + row_lo);  // chunk rows [rlo, rlo + 31] in this warp's lanes
        uint32_t pk[PW / 2];
        if (j0 > rlo + 31) {              // above the diagonal for every row of this warp
#pragma unroll
          for (int q = 0; q < PW / 2; ++q) pk[q] = 0u;
        } else {
          float sv[PW];
          tmem_ldn<PW>(tL + c * PW, sv);
          const int i = rlo + lane;
          const bool full = j0 + PW - 1 <= rlo;  // no masking for any row of this warp
          const float ci = PERSTEP ? T[i] : 0.f;
#pragma unroll
          for (int q = 0; q < PW / 8; ++q) {
            float v[8];
            if (!PERSTEP && full) {
              // gamma^(i-j) = gamma^(i-j0-8q-7) * gamma^(7-e) for j = j0 + 8q + e (pairs)
              const float rf = T[i - j0 - q * 8 - 7];
              const uint64_t rf2 = f2_make(rf, rf);
#pragma unroll
              for (int e = 0; e < 8; e += 2) {
                const uint64_t d2 = f2_mul(rf2, f2_make(T[7 - e], T[6 - e]));
                pk[q * 4 + e / 2] = f2_to_bf2(f2_mul(f2_make(sv[q * 8 + e], sv[q * 8 + e + 1]), d2));
              }
              continue;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int j = j0 + q * 8 + e;
                float dm = 0.f;
                if (j <= i) dm = PERSTEP ? fast_exp(ci - T[j]) : T[i - j];
                v[e] = (j <= i) ? sv[q * 8 + e] * dm : 0.f;
              }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 t2 = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
              pk[q * 4 + e] = *reinterpret_cast<uint32_t*>(&t2);
            }
          }
        }
        if constexpr (PW == 32) tmem_st16_async(tL + pcol(c), pk);
        else tmem_st8_async(tL + pcol(c), pk);
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(B_P);
      if constexpr (late) if (n == n0) {
        // the earlier parts' states from the peers: wait, then R = Dloc R_parts + Rr -> sR
        if (lane == 0) wait_flags(p.wait_flags, p.wait_mask, p.wait_gen, 44);
        __syncwarp();
        acquire_flags(p.wait_flags, p.wait_mask);
        if (f_valid) {
          // four columns at a time (few live registers): state_in, then the parts in order
#pragma unroll
          for (int e = 0; e < EPW / 4; ++e) {
            float4 q4 = p.state_in ? *reinterpret_cast<const float4*>(p.state_in + (size_t)bh * 4096 + f_row * 64 + e0 + 4 * e)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int s = 0; s < p.nprev; ++s) {
              const float Ds = p.prev_D[(size_t)s * p.prev_stride + bh];
              const float4 v = *reinterpret_cast<const float4*>(p.prev_R + (size_t)s * p.prev_stride + (size_t)bh * 4096 +
                                                                f_row * 64 + e0 + 4 * e);
              q4 = make_float4(Ds * q4.x + v.x, Ds * q4.y + v.y, Ds * q4.z + v.z, Ds * q4.w + v.w);
            }
            Rr[4 * e] = fmaf(Dloc, q4.x, Rr[4 * e]);
            Rr[4 * e + 1] = fmaf(Dloc, q4.y, Rr[4 * e + 1]);
            Rr[4 * e + 2] = fmaf(Dloc, q4.z, Rr[4 * e + 2]);
            Rr[4 * e + 3] = fmaf(Dloc, q4.w, Rr[4 * e + 3]);
          }
#pragma unroll
          for (int c = 0; c < EPW / 8; ++c)
            *reinterpret_cast<uint4*>(sR + sw128_chunk(f_row, (e0 >> 3) + c)) = pack16<__nv_bfloat16>(&Rr[c * 8]);
        }
      }
      // the P V products run while k~ and Qs are formed
      // k~ = bf16(phi(k) kdec_j) and Qs = bf16(phi(q) qdec_i) in place (S(n) has read them)
      {
        constexpr int IT = CT * 8 / NTC;
        uint4 kv[IT], qv[IT];
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          kv[it] = reinterpret_cast<const uint4*>(K_)[tid + it * NTC];
          qv[it] = reinterpret_cast<const uint4*>(Q_)[tid + it * NTC];
        }
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          const int idx = tid + it * NTC, row = idx >> 3;
          const float kd = PERSTEP ? fast_exp(T[CT - 1] - T[row]) : T[CT - 1 - row];
          const int qr = q_row(row);  // chunk row of Q tile row `row`
          const float qd = PERSTEP ? fast_exp(T[qr]) : T[qr];
          const uint64_t kd2 = f2_make(kd, kd), qd2 = f2_make(qd, qd);
          uint32_t* wk = reinterpret_cast<uint32_t*>(&kv[it]);
          uint32_t* wq = reinterpret_cast<uint32_t*>(&qv[it]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            wk[i] = f2_to_bf2(f2_mul(bf2_to_f2(wk[i]), kd2));
            wq[i] = f2_to_bf2(f2_mul(bf2_to_f2(wq[i]), qd2));
          }
          reinterpret_cast<uint4*>(K_)[idx] = kv[it];
          reinterpret_cast<uint4*>(Q_)[idx] = qv[it];
        }
      }
      fence_proxy_async_smem();
      warp_arrive(B_KQ);
      // during the products: the outputs of the previous chunk, then the next chunk's phi
      if (n > n0 && !gn_gate(n - 1)) { ok = false; break; }
      if (n + 1 < n1 && !prep(n + 1, nxt)) { ok = false; break; }
      if (!mbar_wait_warp(&bars[B_Y], yph, 60)) { ok = false; break; }
      yph ^= 1;
      tc_fence_after();
      // Y of both row blocks and U out of TMEM (one wait); then S(n+1) may overwrite them
      float yv2[2][EPW], u[EPW];
      tmem_ld16x3(tL + YCOL + e0, tL + YCOL + 64 + e0, tL + UCOL + e0, yv2[0], yv2[1], u);
      tc_fence_before();
      if (n + 1 < n1) warp_arrive(B_READY);
      // y = bf16(Y) (y_slot is bf16), kept as bf16 pairs for the deferred GroupNorm; partials
      float2* red = sRed + (size_t)cur * (NWG * CT);
#pragma unroll
      for (int rb = 0; rb < 2; ++rb) {
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int e = 0; e < EPW; e += 2) {
          yp[rb][e / 2] = f2_to_bf2(f2_make(yv2[rb][e], yv2[rb][e + 1]));
          float lo, hi;
          f2_split(bf2_to_f2(yp[rb][e / 2]), lo, hi);
          s1 += lo + hi;
          s2 = fmaf(lo, lo, fmaf(hi, hi, s2));
        }
        red[wg * CT + rb * RB + my_row] = make_float2(s1, s2);
      }
      // R <- gC R + U (fp32) -> sR (bf16) for the next chunk's Qs R (issued after KQ(n+1))
      {
        const float gC = PERSTEP ? fast_exp(T[CT]) : T[CT];
#pragma unroll
        for (int e = 0; e < EPW; ++e) Rr[e] = fmaf(Rr[e], gC, u[e]);
        if (f_valid) {
#pragma unroll
          for (int c = 0; c < EPW / 8; ++c)
            *reinterpret_cast<uint4*>(sR + sw128_chunk(f_row, (e0 >> 3) + c)) = pack16<__nv_bfloat16>(&Rr[c * 8]);
        }
      }
      fence_proxy_async_smem();
      // this warp's GroupNorm partials of chunk n (and warp 0's table of chunk n+1) are in place
      warp_arrive(B_SYNC);
    }
    if (ok && n0 < n1) ok = gn_gate(n1 - 1);
    if (ok && seg == p.nseg - 1 && p.state_out && f_valid) {
      float* dst = p.state_out + (size_t)bh * 4096 + f_row * 64 + e0;
#pragma unroll
      for (int e = 0; e < EPW; e += 4)
        *reinterpret_cast<float4*>(dst + e) = make_float4(Rr[e], Rr[e + 1], Rr[e + 2], Rr[e + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

int slot_make_map(CUtensorMap* m, const void* base, int64_t width, int64_t L, int64_t B, int64_t row_stride,
                    int64_t batch_stride, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(HDC_E_SHAPE, "slot_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)L, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2, (cuuint64_t)batch_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HDC_E_SHAPE, "slot_tc: tensor map encode failed (%d)", (int)r);
  return 0;
}

static int make_map(CUtensorMap* m, const void* base, int64_t width, int64_t L, int64_t B, int64_t row_stride,
                    int64_t batch_stride, int box_rows) {
  return slot_make_map(m, base, width, L, B, row_stride, batch_stride, box_rows);
}

template <int CT>
static size_t smem_out_bytes() {
  return 1024 + OutCfg<CT>::NST * 3 * CT * 128 + OutCfg<CT>::PBYTES + 64 * 128 +
         (CT + 4 + 128 + CT * OutCfg<CT>::SRED) * 4 + 6 * 8 + 16;
}
static size_t smem_state_bytes(int CT) { return 1024 + 4 * CT * 128 + (CT + 4) * 4 + 64; }

// pass A: the warp-specialized kernel for chunk 256, the lock-step one otherwise
template <int CT, bool PS>
static int launch_state(const CUtensorMap& mk, const CUtensorMap& mv, const SlotTcParams& p, unsigned grid,
                        cudaStream_t s) {
  if constexpr (CT == 256) {
    cudaFuncSetAttribute(slot_tc_state_pipe_kernel<PS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)spipe::SMEM);
    slot_tc_state_pipe_kernel<PS><<<grid, spipe::NT, spipe::SMEM, s>>>(mk, mv, p);
    return launch_status("slot_tc_state_pipe_kernel");
  } else {
    const size_t sm = smem_state_bytes(CT);
    cudaFuncSetAttribute(slot_tc_state_kernel<CT, PS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    slot_tc_state_kernel<CT, PS><<<grid, kStateThreads, sm, s>>>(mk, mv, p);
    return launch_status("slot_tc_state_kernel");
  }
}

// One output CTA per SM for chunk 128 / 256 (512 TMEM columns), two for chunk 64.
static void plan_segments(int64_t BH, int N, int C, int* nseg, int* seg_len) {
  const int slots = num_sms() * (C == 64 ? 2 : 1);
  int s = (int)(slots / BH);
  if (s < 1) s = 1;
  if (s > N) s = N;
  int len = (N + s - 1) / s;
  *seg_len = len;
  *nseg = (N + len - 1) / len;
}

size_t slot_tc_workspace(int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C) {
  int nseg, len;
  plan_segments(B * H, (int)(L / C), (int)C, &nseg, &len);
  if (C == 64 && (L / C) % 4 == 0) {  // the four-chunk kernels' plan (slot_mc.cu)
    int nseg_mc, len_mc, split;
    slot_mc_plan(B * H, (int)(L / C), &nseg_mc, &len_mc, &split);
    nseg_mc *= split;  // pass A's pieces (the workspace holds one state per piece)
    nseg = nseg_mc > nseg ? nseg_mc : nseg;
  }
  return (size_t)(B * H) * nseg * (4096 + 1) * sizeof(float) + 256;
}

bool slot_tc_supported(const SlotParams& p, int64_t B, int64_t in_sb, int64_t in_st) {
  if (p.bd != 64 || p.hd % 8 != 0) return false;
  if (p.C != 64 && p.C != 128 && p.C != 256) return false;
  if (p.rows != p.C) return false;
  if (in_st % 8 != 0 || (B > 1 && in_sb % 8 != 0) || in_st < (int64_t)p.H * p.hd) return false;
  if ((int64_t)p.H * p.hd < 64) return false;  // the TMA box is 64 columns wide
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v)) return false;
  return true;
}

// Lane s waits (bounded) for flags[s] to reach *gen, for every bit s of mask.
__global__ void slot_wait_kernel(const uint32_t* flags, uint32_t mask, const uint32_t* gen) {
  const int s = threadIdx.x;
  if ((mask >> s) & 1u) wait_flag(flags + s, *gen, 44);
}

template <int CT, bool PS, bool GATE>
static int run_tc(const SlotParams& sp, const SlotGate* gt, const SlotCarry* carry, int64_t B, int64_t in_sb,
                  int64_t in_st, void* ws, cudaStream_t s) {
  // chunk 64 without the gate epilogue: four chunks per CTA iteration
  if constexpr (CT == 64 && !GATE) {
    if (!carry && slot_mc_supported(sp)) return slot_mc_fwd(sp, B, in_sb, in_st, ws, s);
  }
  const int64_t BH = B * sp.H;
  SlotTcParams p{};
  p.gamma = sp.gamma; p.log_a = sp.log_a; p.y = sp.y; p.y_sb = sp.y_sb; p.y_sh = sp.y_sh; p.y_st = sp.y_st;
  p.state_in = sp.state_in; p.state_out = sp.state_out;
  p.L = sp.L; p.H = sp.H; p.hd = sp.hd; p.N = sp.N;
  if (gt) {
    p.gate = gt->gate; p.g_sb = gt->g_sb; p.g_st = gt->g_st; p.gn_w = gt->gn_w; p.gn_b = gt->gn_b;
  }
  plan_segments(BH, sp.N, sp.C, &p.nseg, &p.seg_len);
  p.Rseg = static_cast<float*>(ws);
  p.Dseg = p.Rseg + (size_t)BH * p.nseg * 4096;
  p.y_vec = (aligned16(sp.y) && sp.y_sb % 8 == 0 && sp.y_sh % 8 == 0 && sp.y_st % 8 == 0 && sp.hd % 8 == 0) ? 1 : 0;
  const int64_t W = (int64_t)sp.H * sp.hd;
  CUtensorMap mq, mk, mv;
  const int64_t sb = B > 1 ? in_sb : (int64_t)sp.L * in_st;
  if (int e = make_map(&mq, sp.q, W, sp.L, B, in_st, sb, CT)) return e;
  if (int e = make_map(&mk, sp.k, W, sp.L, B, in_st, sb, CT)) return e;
  if (int e = make_map(&mv, sp.v, W, sp.L, B, in_st, sb, CT)) return e;
  if (carry) {
    p.prev_R = carry->prev_R; p.prev_D = carry->prev_D; p.prev_stride = carry->prev_stride; p.nprev = carry->nprev;
    p.wait_flags = carry->wait_flags; p.wait_mask = carry->wait_mask; p.wait_gen = carry->wait_gen;
  }
  // with a carry the workspace already holds every segment's state (hdc_slot_state_fwd)
  if (p.nseg > 1 && !carry) {
    p.nseg_a = p.nseg - 1;
    if (int e = launch_state<CT, PS>(mk, mv, p, (unsigned)(BH * p.nseg_a), s)) return e;
  }
  // chunk 256 with the fused gate and head_dim 64: the warp-specialized kernel, when a
  // head's 64 columns of the gate and of the outputs are contiguous and 16-byte aligned
  // (gate tile in by TMA, one TMA store of the gated outputs per chunk)
  if constexpr (CT == 256 && GATE) {
    const bool pipe_ok = sp.hd == 64 && sp.y_sh == 64 && aligned16(sp.y) && sp.y_st % 8 == 0 &&
                         (B == 1 || sp.y_sb % 8 == 0) && aligned16(gt->gate) && gt->g_st % 8 == 0 &&
                         (B == 1 || gt->g_sb % 8 == 0) && aligned16(gt->gn_w) && aligned16(gt->gn_b);
    if (pipe_ok) {
      SlotPipeMaps mg{};
      if (int e = make_map(&mg.gate, gt->gate, W, sp.L, B, gt->g_st, B > 1 ? gt->g_sb : (int64_t)sp.L * gt->g_st, CT))
        return e;
      if (int e = make_map(&mg.out, sp.y, W, sp.L, B, sp.y_st, B > 1 ? sp.y_sb : (int64_t)sp.L * sp.y_st, CT))
        return e;
      CUtensorMap mq32;  // Q in 32-row boxes (row block 0 is loaded in permuted block order)
      if (int e = make_map(&mq32, sp.q, W, sp.L, B, in_st, sb, 32)) return e;
      const size_t sm = pipe::SMEM;
      // right after the state pass: a programmatic dependent launch, so that output CTAs
      // take the SMs as state CTAs leave them and overlap their first chunk's loads, phi and
      // S with the end of the state pass (the kernel waits before it reads the states)
      const bool after_state = p.nseg > 1 && !carry;
      auto go = [&](auto kernel) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)(BH * p.nseg));
        cfg.blockDim = dim3(pipe::NT);
        cfg.dynamicSmemBytes = sm;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = after_state ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, kernel, mq32, mk, mv, mg, p);
      };
      const cudaError_t le = p.wait_mask ? go(slot_tc_pipe_kernel<PS, true>) : go(slot_tc_pipe_kernel<PS, false>);
      if (le != cudaSuccess) return fail((int)le, "slot_tc_pipe_kernel launch: %s", cudaGetErrorString(le));
      return launch_status("slot_tc_pipe_kernel");
    }
  }
  if (p.wait_mask) {  // the lock-step kernel reads the earlier parts at its start: wait first
    slot_wait_kernel<<<1, 32, 0, s>>>(p.wait_flags, p.wait_mask, p.wait_gen);
    if (int e = launch_status("slot_wait_kernel")) return e;
  }
  const size_t sm = smem_out_bytes<CT>();
  cudaFuncSetAttribute(slot_tc_out_kernel<CT, PS, GATE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  slot_tc_out_kernel<CT, PS, GATE><<<(unsigned)(BH * p.nseg), OutCfg<CT>::NT, sm, s>>>(mq, mk, mv, p);
  return launch_status("slot_tc_out_kernel");
}

// Fold the segment states of each (batch, head) into the state after the whole sequence
// (from zero) and the product of all chunk decays.
__global__ void __launch_bounds__(256) slot_fold_kernel(SlotTcParams p) {
  const int bh = blockIdx.x;
  float R[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) R[e] = 0.f;
  float D = 1.f;
  // (unrolled so that the loads of several segments are in flight together)
#pragma unroll 4
  for (int s = 0; s < p.nseg; ++s) {
    const float Ds = p.Dseg[(size_t)bh * p.nseg + s];
    const float4* src = reinterpret_cast<const float4*>(p.Rseg + ((size_t)bh * p.nseg + s) * 4096 + threadIdx.x * 16);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 v = src[e];
      R[4 * e] = Ds * R[4 * e] + v.x;
      R[4 * e + 1] = Ds * R[4 * e + 1] + v.y;
      R[4 * e + 2] = Ds * R[4 * e + 2] + v.z;
      R[4 * e + 3] = Ds * R[4 * e + 3] + v.w;
    }
    D *= Ds;
  }
  float* dst = p.state_out + (size_t)bh * 4096 + threadIdx.x * 16;
#pragma unroll
  for (int e = 0; e < 16; ++e) dst[e] = R[e];
  if (threadIdx.x == 0 && p.y) static_cast<float*>(p.y)[bh] = D;
}

template <int CT, bool PS>
static int run_tc_state(const SlotParams& sp, int64_t B, int64_t in_sb, int64_t in_st, void* ws, float* decay_out,
                        cudaStream_t s) {
  const int64_t BH = B * sp.H;
  SlotTcParams p{};
  p.gamma = sp.gamma; p.log_a = sp.log_a; p.state_out = sp.state_out; p.y = decay_out;
  p.L = sp.L; p.H = sp.H; p.hd = sp.hd; p.N = sp.N;
  plan_segments(BH, sp.N, sp.C, &p.nseg, &p.seg_len);
  p.nseg_a = p.nseg;
  p.Rseg = static_cast<float*>(ws);
  p.Dseg = p.Rseg + (size_t)BH * p.nseg * 4096;
  const int64_t W = (int64_t)sp.H * sp.hd;
  CUtensorMap mk, mv;
  const int64_t sb = B > 1 ? in_sb : (int64_t)sp.L * in_st;
  if (int e = make_map(&mk, sp.k, W, sp.L, B, in_st, sb, CT)) return e;
  if (int e = make_map(&mv, sp.v, W, sp.L, B, in_st, sb, CT)) return e;
  if (int e = launch_state<CT, PS>(mk, mv, p, (unsigned)(BH * p.nseg), s)) return e;
  slot_fold_kernel<<<(unsigned)BH, 256, 0, s>>>(p);
  return launch_status("slot_fold_kernel");
}

int slot_tc_state_fwd(const SlotParams& p, int64_t B, int64_t in_sb, int64_t in_st, void* ws, float* decay_out,
                      cudaStream_t s) {
  const bool ps = p.log_a != nullptr;
  switch (p.C) {
    case 64: return ps ? run_tc_state<64, true>(p, B, in_sb, in_st, ws, decay_out, s)
                       : run_tc_state<64, false>(p, B, in_sb, in_st, ws, decay_out, s);
    case 128: return ps ? run_tc_state<128, true>(p, B, in_sb, in_st, ws, decay_out, s)
                        : run_tc_state<128, false>(p, B, in_sb, in_st, ws, decay_out, s);
    default: return ps ? run_tc_state<256, true>(p, B, in_sb, in_st, ws, decay_out, s)
                       : run_tc_state<256, false>(p, B, in_sb, in_st, ws, decay_out, s);
  }
}

template <bool GATE>
static int slot_tc_dispatch(const SlotParams& p, const SlotGate* gt, const SlotCarry* cy, int64_t B, int64_t in_sb,
                            int64_t in_st, void* ws, cudaStream_t s) {
  const bool ps = p.log_a != nullptr;
  switch (p.C) {
    case 64:
      return ps ? run_tc<64, true, GATE>(p, gt, cy, B, in_sb, in_st, ws, s)
                : run_tc<64, false, GATE>(p, gt, cy, B, in_sb, in_st, ws, s);
    case 128:
      return ps ? run_tc<128, true, GATE>(p, gt, cy, B, in_sb, in_st, ws, s)
                : run_tc<128, false, GATE>(p, gt, cy, B, in_sb, in_st, ws, s);
    default:
      return ps ? run_tc<256, true, GATE>(p, gt, cy, B, in_sb, in_st, ws, s)
                : run_tc<256, false, GATE>(p, gt, cy, B, in_sb, in_st, ws, s);
  }
}

int slot_tc_fwd(const SlotParams& p, const SlotGate* gt, const SlotCarry* carry, int64_t B, int64_t in_sb,
                int64_t in_st, void* ws, cudaStream_t s) {
  return gt ? slot_tc_dispatch<true>(p, gt, carry, B, in_sb, in_st, ws, s)
            : slot_tc_dispatch<false>(p, gt, carry, B, in_sb, in_st, ws, s);
}

}  // namespace hdc
