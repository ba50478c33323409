// Peer-memory exchange for sequence parallelism over NVLink / NVSwitch, sm_100a.
//
// One process per GPU.  Every rank allocates one mailbox (hdc_peer_alloc) and shares it
// with the other ranks through CUDA IPC (hdc_ipc_handle / hdc_ipc_open).  A producer then
// stores its data straight into the consumers' mailboxes over NVLink (plain 16-byte peer
// stores, no multicast) and raises a flag there; a consumer waits for the flags it needs
// (bounded spins) before the kernels that read the data run.  This replaces a collective
// where the data flow is one-directional: under sequence parallelism rank r only needs the
// carries of ranks < r and the halo rows of rank r - 1.
//
// Flags carry a generation number: every rank bumps its own device counter once per
// forward (hdc_peer_gen_bump) and all ranks run the same forwards, so a consumer waits for
// its own generation (or a later one) and no flag ever needs clearing.  A flag barrier at the end of
// each forward (hdc_peer_barrier) keeps a rank from writing a mailbox region of the next
// forward while a slower rank still reads the current one.
//
// Memory ordering: the producer CTA's threads store the data, then __syncthreads(), then one
// thread issues fence.acq_rel.sys and a relaxed system-scope flag store (the fence is
// cumulative over the CTA's stores observed through the barrier).  The consumer loads the
// flag with ld.acquire.sys; the kernels that read the data follow in stream order.
//
// Every wait gives up after ~2 s of %globaltimer, records an error code readable through
// hdc_device_error() and returns, so a missing peer can not hang the GPU.
#include <algorithm>
#include <cstring>

#include "flag.cuh"

namespace hdc {

// CTAs [kc t, kc t + kc) copy `bytes` from src to dst_base[t] + dst_off, one slice each;
// the CTA that completes target t's last slice (counted in counters[t], zero between calls)
// sets flag_base[t] + flag_off to the generation.  Targets t with bit t of `mask` clear are
// skipped.  Ordering: every CTA's stores, its system-scope fence, then its count; the last
// CTA's count, its fence, then the flag (fence - atomic / atomic - fence synchronisation),
// so a consumer that acquires the flag sees every slice.
__global__ void __launch_bounds__(512) peer_put_kernel(const uint4* src, size_t n16, const uint64_t* dst_base,
                                                       uint64_t dst_off, uint64_t flag_off, uint32_t mask,
                                                       const uint32_t* gen, uint32_t* counters, int kc) {
  const int t = blockIdx.x / kc, c = blockIdx.x - t * kc;
  if (!((mask >> t) & 1u)) return;
  uint4* dst = reinterpret_cast<uint4*>(dst_base[t] + dst_off);
  const size_t lo = n16 * (size_t)c / kc, hi = n16 * (size_t)(c + 1) / kc;
  // eight loads in flight per thread before their stores
  for (size_t i0 = lo; i0 < hi; i0 += 8 * (size_t)blockDim.x) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const size_t i = i0 + (size_t)k * blockDim.x + threadIdx.x;
      if (i < hi) v[k] = src[i];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const size_t i = i0 + (size_t)k * blockDim.x + threadIdx.x;
      if (i < hi) dst[i] = v[k];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    if (kc == 1 || atomicAdd(&counters[t], 1u) == (uint32_t)(kc - 1)) {
      if (kc > 1) {
        counters[t] = 0;  // the next call on this counter array comes after this kernel
        fence_acq_rel_sys();
      }
      st_relaxed_sys(reinterpret_cast<uint32_t*>(dst_base[t] + flag_off), *gen);
    }
  }
}

// lane s waits for flags[s] == *gen for every bit s of mask (s < 32), each wait bounded by
// limit_ns
__global__ void peer_wait_kernel(const uint32_t* flags, uint32_t mask, const uint32_t* gen, uint64_t limit_ns) {
  const int s = threadIdx.x;
  if (s < 32 && ((mask >> s) & 1u)) wait_flag(flags + s, *gen, 41, limit_ns);
}

__global__ void peer_gen_bump_kernel(uint32_t* gen) { *gen += 1; }

// every rank writes its generation into slot `rank` of every rank's barrier array, then
// waits until all `world` slots of its own array hold its generation
__global__ void peer_barrier_kernel(const uint64_t* base, uint64_t bar_off, int world, int rank,
                                    const uint32_t* local_bar, const uint32_t* gen) {
  const int s = threadIdx.x;
  const uint32_t g = *gen;
  if (s < world) {
    fence_acq_rel_sys();
    st_relaxed_sys(reinterpret_cast<uint32_t*>(base[s] + bar_off) + rank, g);
  }
  __syncwarp();
  if (s < world) wait_flag(local_bar + s, g, 42);
}

}  // namespace hdc

using namespace hdc;

extern "C" int hdc_peer_alloc(size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return fail(HDC_E_NULL, "peer_alloc: null output or zero bytes");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail((int)e, "peer_alloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can map it
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail((int)e, "peer_alloc: %s", cudaGetErrorString(e));
  }
  *dev_ptr = p;
  return 0;
}

extern "C" int hdc_peer_free(void* dev_ptr) {
  const cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? 0 : fail((int)e, "peer_free: %s", cudaGetErrorString(e));
}

extern "C" int hdc_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int hdc_ipc_handle(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return fail(HDC_E_NULL, "ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return fail((int)e, "ipc_handle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

extern "C" int hdc_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(HDC_E_NULL, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? 0 : fail((int)e, "ipc_open: %s", cudaGetErrorString(e));
}

extern "C" int hdc_ipc_close(void* dev_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? 0 : fail((int)e, "ipc_close: %s", cudaGetErrorString(e));
}

extern "C" int hdc_peer_put(const void* src, size_t bytes, const uint64_t* dst_base, uint64_t dst_off,
                            uint64_t flag_off, uint32_t mask, int world, const uint32_t* gen,
                            uint32_t* counters, hdc_stream_t stream) {
  if (!src || !dst_base || !gen || !counters) return fail(HDC_E_NULL, "peer_put: null pointer");
  if (world < 1 || world > 32) return fail(HDC_E_SHAPE, "peer_put: world %d (1..32)", world);
  if (bytes % 16 || !aligned16(src) || dst_off % 16 || flag_off % 4)
    return fail(HDC_E_ALIGN, "peer_put: src / dst must be 16-byte aligned and sizes multiples of 16");
  if (mask == 0) return 0;
  // one CTA per 8 KB slice of a target's copy (at most 64): each CTA's stores, then its
  // system-scope fence, run in parallel with the other slices' instead of one SM pushing
  // the whole copy and then waiting for it
  const int kc = (int)std::min<size_t>(64, std::max<size_t>(1, (bytes + 8191) / 8192));
  peer_put_kernel<<<world * kc, 512, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), bytes / 16, dst_base, dst_off, flag_off, mask, gen, counters, kc);
  return launch_status("peer_put_kernel");
}

extern "C" int hdc_peer_wait_for(const uint32_t* flags, uint32_t mask, const uint32_t* gen, uint64_t timeout_ns,
                                 hdc_stream_t stream) {
  if (!flags || !gen) return fail(HDC_E_NULL, "peer_wait: null pointer");
  if (timeout_ns == 0 || timeout_ns > kPeerWaitNs)
    return fail(HDC_E_SHAPE, "peer_wait: timeout %llu ns (1 .. 2e9)", (unsigned long long)timeout_ns);
  if (mask == 0) return 0;
  peer_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, mask, gen, timeout_ns);
  return launch_status("peer_wait_kernel");
}

extern "C" int hdc_peer_wait(const uint32_t* flags, uint32_t mask, const uint32_t* gen, hdc_stream_t stream) {
  return hdc_peer_wait_for(flags, mask, gen, kPeerWaitNs, stream);
}

extern "C" int hdc_peer_gen_bump(uint32_t* gen, hdc_stream_t stream) {
  if (!gen) return fail(HDC_E_NULL, "peer_gen_bump: null pointer");
  peer_gen_bump_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(gen);
  return launch_status("peer_gen_bump_kernel");
}

extern "C" int hdc_peer_barrier(const uint64_t* base, uint64_t bar_off, int world, int rank,
                                const uint32_t* local_bar, const uint32_t* gen, hdc_stream_t stream) {
  if (!base || !local_bar || !gen) return fail(HDC_E_NULL, "peer_barrier: null pointer");
  if (world < 1 || world > 32 || rank < 0 || rank >= world || bar_off % 4)
    return fail(HDC_E_SHAPE, "peer_barrier: world %d rank %d", world, rank);
  peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(base, bar_off, world, rank,
                                                                            local_bar, gen);
  return launch_status("peer_barrier_kernel");
}
