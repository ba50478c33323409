// Device timestamps for tracing the layer's launch sequence (hdcmamba_b200/trace.py).
//
// hdc_trace_stamp enqueues a one-thread kernel that writes %globaltimer (ns) into a device
// array slot, so stamps taken between the launches of a CUDA graph time every op of the
// graph on the device, in stream order, without host involvement.
#include "common.cuh"

namespace hdc {

__global__ void trace_stamp_kernel(unsigned long long* buf, long long index) {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  buf[index] = t;
}

}  // namespace hdc

extern "C" int hdc_trace_stamp(unsigned long long* buf, long long index, hdc_stream_t stream) {
  if (!buf) return hdc::fail(HDC_E_NULL, "trace_stamp: null buffer");
  if (index < 0) return hdc::fail(HDC_E_SHAPE, "trace_stamp: index %lld", index);
  hdc::trace_stamp_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(buf, index);
  return hdc::launch_status("trace_stamp_kernel");
}
