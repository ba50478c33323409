// hdc_slot_scan_fwd: argument checks and dispatch between the tcgen05 kernel
// (bf16 activations) and the CUDA-core kernel (fp32 activations).
#include "slot.cuh"

using namespace hdc;

extern "C" size_t hdc_slot_workspace_bytes(int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C) {
  if (B < 1 || H < 1 || hd < 1 || C < 1 || L < C) return 0;
  const size_t a = slot_simt_workspace(B, L, H, hd, C), b = slot_tc_workspace(B, L, H, hd, C);
  return a > b ? a : b;
}

// Shared body of hdc_slot_scan_fwd / hdc_slot_scan_fwd_path: `path` 0 automatic, 1 CUDA
// cores, 2 tcgen05 required; *path_used (when non-NULL) receives 1 for tcgen05, 0 for CUDA
// cores.  No state outlives the call.
extern "C" int hdc_slot_scan_fwd_path(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                                      int64_t in_st, const void* gamma, const float* log_a, void* y, int64_t y_sb,
                                      int64_t y_sh, int64_t y_st, const float* state_in, float* state_out,
                                      void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                                      int64_t hd, int64_t C, int64_t rows, int path, int* path_used,
                                      hdc_stream_t stream) {
  if (path < 0 || path > 2) return fail(HDC_E_SHAPE, "slot: path %d (0 auto, 1 CUDA cores, 2 tcgen05)", path);
  if (dtype != HDC_F32 && dtype != HDC_BF16) return fail(HDC_E_DTYPE, "slot: dtype %d", dtype);
  if (!q || !k || !v || !y || !workspace || (!gamma && !log_a)) return fail(HDC_E_NULL, "slot: null pointer");
  if (B < 1 || H < 1 || hd < 1 || hd > 128 || C < 1 || C > 256 || L < C || L % C != 0)
    return fail(HDC_E_SHAPE, "slot: B=%lld L=%lld H=%lld hd=%lld C=%lld (hd <= 128, C <= 256, L %% C == 0)",
                (long long)B, (long long)L, (long long)H, (long long)hd, (long long)C);
  if (rows < 1 || rows > C || (log_a && rows != C)) return fail(HDC_E_SHAPE, "slot: rows=%lld", (long long)rows);
  const size_t need = hdc_slot_workspace_bytes(B, L, H, hd, C);
  if (workspace_bytes < need)
    return fail(HDC_E_WORKSPACE, "slot: workspace %zu < %zu bytes", workspace_bytes, need);
  SlotParams p{};
  p.q = q; p.k = k; p.v = v; p.in_sb = in_sb; p.in_st = in_st; p.gamma = gamma; p.log_a = log_a;
  p.y = y; p.y_sb = y_sb; p.y_sh = y_sh; p.y_st = y_st; p.state_in = state_in; p.state_out = state_out;
  p.L = (int)L; p.H = (int)H; p.hd = (int)hd; p.C = (int)C; p.rows = (int)rows; p.N = (int)(L / C);
  p.bd = (int)feature_block(hd);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const bool tc = dtype == HDC_BF16 && path != 1 && slot_tc_supported(p, B, in_sb, in_st);
  if (path == 2 && !tc) return fail(HDC_E_SHAPE, "slot: tcgen05 path required but not applicable");
  if (path_used) *path_used = tc ? 1 : 0;
  return tc ? slot_tc_fwd(p, nullptr, nullptr, B, in_sb, in_st, workspace, s) : slot_simt_fwd(dtype, p, B, workspace, s);
}

extern "C" int hdc_slot_scan_fwd(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                                 int64_t in_st, const void* gamma, const float* log_a, void* y, int64_t y_sb,
                                 int64_t y_sh, int64_t y_st, const float* state_in, float* state_out,
                                 void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                                 int64_t hd, int64_t C, int64_t rows, hdc_stream_t stream) {
  return hdc_slot_scan_fwd_path(dtype, q, k, v, in_sb, in_st, gamma, log_a, y, y_sb, y_sh, y_st, state_in,
                                state_out, workspace, workspace_bytes, B, L, H, hd, C, rows, 0, nullptr, stream);
}

static int slot_gate_common(const char* who, const void* q, const void* k, const void* v, int64_t in_sb,
                            int64_t in_st, const void* gamma, const float* log_a, const void* gate, int64_t gate_sb,
                            int64_t gate_st, const void* gn_w, const void* gn_b, void* out, int64_t out_sb,
                            int64_t out_sh, int64_t out_st, const float* state_in, float* state_out,
                            void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H, int64_t hd,
                            int64_t C, const SlotCarry* carry, cudaStream_t stream) {
  if (!q || !k || !v || !out || !gate || !gn_w || !gn_b || !workspace || (!gamma && !log_a))
    return fail(HDC_E_NULL, "%s: null pointer", who);
  if (B < 1 || H < 1 || hd < 1 || hd > 64 || C < 1 || L < C || L % C != 0)
    return fail(HDC_E_SHAPE, "%s: B=%lld L=%lld H=%lld hd=%lld C=%lld", who, (long long)B, (long long)L,
                (long long)H, (long long)hd, (long long)C);
  const size_t need = hdc_slot_workspace_bytes(B, L, H, hd, C);
  if (workspace_bytes < need)
    return fail(HDC_E_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, need);
  if (!aligned16(out) || !aligned16(gate) || out_sb % 8 || out_sh % 8 || out_st % 8 || gate_sb % 8 || gate_st % 8)
    return fail(HDC_E_ALIGN, "%s: out / gate need 16-byte aligned rows", who);
  SlotParams p{};
  p.q = q; p.k = k; p.v = v; p.in_sb = in_sb; p.in_st = in_st; p.gamma = gamma; p.log_a = log_a;
  p.y = out; p.y_sb = out_sb; p.y_sh = out_sh; p.y_st = out_st; p.state_in = state_in; p.state_out = state_out;
  p.L = (int)L; p.H = (int)H; p.hd = (int)hd; p.C = (int)C; p.rows = (int)C; p.N = (int)(L / C);
  p.bd = (int)feature_block(hd);
  if (!slot_tc_supported(p, B, in_sb, in_st))
    return fail(HDC_E_SHAPE, "%s: the fused epilogue needs the tcgen05 path (head_dim %% 8 == 0, "
                "chunk 64/128/256, aligned row-major q/k/v)", who);
  SlotGate g{gate, gate_sb, gate_st, gn_w, gn_b};
  return slot_tc_fwd(p, &g, carry, B, in_sb, in_st, workspace, stream);
}

extern "C" int hdc_slot_gate_fwd(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                                 int64_t in_st, const void* gamma, const float* log_a, const void* gate,
                                 int64_t gate_sb, int64_t gate_st, const void* gn_w, const void* gn_b, void* out,
                                 int64_t out_sb, int64_t out_sh, int64_t out_st, const float* state_in,
                                 float* state_out, void* workspace, size_t workspace_bytes, int64_t B, int64_t L,
                                 int64_t H, int64_t hd, int64_t C, hdc_stream_t stream) {
  if (dtype != HDC_BF16) return fail(HDC_E_DTYPE, "slot_gate: bf16 activations only");
  return slot_gate_common("slot_gate", q, k, v, in_sb, in_st, gamma, log_a, gate, gate_sb, gate_st, gn_w, gn_b,
                          out, out_sb, out_sh, out_st, state_in, state_out, workspace, workspace_bytes, B, L, H,
                          hd, C, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int hdc_slot_gate_carry_fwd(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                                       int64_t in_st, const void* gamma, const float* log_a, const void* gate,
                                       int64_t gate_sb, int64_t gate_st, const void* gn_w, const void* gn_b,
                                       void* out, int64_t out_sb, int64_t out_sh, int64_t out_st,
                                       const float* prev_state, const float* prev_decay, int64_t prev_stride,
                                       int64_t n_prev, float* state_out, void* workspace, size_t workspace_bytes,
                                       int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C,
                                       const uint32_t* wait_flags, uint32_t wait_mask, const uint32_t* wait_gen,
                                       hdc_stream_t stream) {
  if (wait_mask && (!wait_flags || !wait_gen)) return fail(HDC_E_NULL, "slot_gate_carry: wait_mask needs flags and gen");
  if (dtype != HDC_BF16) return fail(HDC_E_DTYPE, "slot_gate_carry: bf16 activations only");
  if (n_prev < 0 || (n_prev > 0 && (!prev_state || !prev_decay)))
    return fail(HDC_E_NULL, "slot_gate_carry: n_prev=%lld needs prev_state / prev_decay", (long long)n_prev);
  if (n_prev > 1 && prev_stride < B * H * 4096)
    return fail(HDC_E_SHAPE, "slot_gate_carry: prev_stride %lld < B*H*4096", (long long)prev_stride);
  if (n_prev > 0 && (!aligned16(prev_state) || prev_stride % 4 != 0))
    return fail(HDC_E_ALIGN, "slot_gate_carry: prev_state must be 16-byte aligned, prev_stride a multiple of 4");
  const SlotCarry cy{prev_state, prev_decay, prev_stride, (int)n_prev, wait_flags, wait_mask, wait_gen};
  return slot_gate_common("slot_gate_carry", q, k, v, in_sb, in_st, gamma, log_a, gate, gate_sb, gate_st, gn_w,
                          gn_b, out, out_sb, out_sh, out_st, nullptr, state_out, workspace, workspace_bytes, B, L,
                          H, hd, C, &cy, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int hdc_slot_state_fwd(int dtype, const void* k, const void* v, int64_t in_sb, int64_t in_st,
                                  const void* gamma, const float* log_a, float* state_out, float* decay_out,
                                  void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                                  int64_t hd, int64_t C, hdc_stream_t stream) {
  if (dtype != HDC_BF16) return fail(HDC_E_DTYPE, "slot_state: bf16 activations only");
  if (!k || !v || !state_out || !decay_out || !workspace || (!gamma && !log_a))
    return fail(HDC_E_NULL, "slot_state: null pointer");
  if (B < 1 || H < 1 || hd < 1 || hd > 64 || C < 1 || L < C || L % C != 0)
    return fail(HDC_E_SHAPE, "slot_state: B=%lld L=%lld H=%lld hd=%lld C=%lld", (long long)B, (long long)L,
                (long long)H, (long long)hd, (long long)C);
  const size_t need = hdc_slot_workspace_bytes(B, L, H, hd, C);
  if (workspace_bytes < need)
    return fail(HDC_E_WORKSPACE, "slot_state: workspace %zu < %zu bytes", workspace_bytes, need);
  SlotParams p{};
  p.q = k; p.k = k; p.v = v; p.in_sb = in_sb; p.in_st = in_st; p.gamma = gamma; p.log_a = log_a;
  p.state_out = state_out;
  p.L = (int)L; p.H = (int)H; p.hd = (int)hd; p.C = (int)C; p.rows = (int)C; p.N = (int)(L / C);
  p.bd = (int)feature_block(hd);
  if (!slot_tc_supported(p, B, in_sb, in_st))
    return fail(HDC_E_SHAPE, "slot_state: needs the tcgen05 path (head_dim %% 8 == 0, chunk 64/128/256)");
  return slot_tc_state_fwd(p, B, in_sb, in_st, workspace, decay_out, reinterpret_cast<cudaStream_t>(stream));
}
