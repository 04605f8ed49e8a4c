// illumina_op_dwpw_noalloc: the fused depthwise -> pointwise entry point for
// callers that must not allocate device memory.
//
// illumina_op_dwpw repacks the caller's [C][k][k] depthwise weights into the
// kernel's [k*k][C] layout in a temporary buffer from cudaMallocAsync. This
// variant repacks into a fixed, file-scope device array instead, so the call
// performs no allocation of any kind: it only launches the repack kernel and
// the fused dw->pw kernel. It always runs the SIMT engine's kernel (k_gemm),
// whatever illumina_set_op_engine selected: the tensor engine would need its
// weight images in an allocation.
//
// The array belongs to every GPU that loads this library and stays reserved
// until the process exits. Every call on a device shares it and it keeps the
// previous call's contents; each call overwrites the in_c*k*k floats it uses
// before reading them, so nothing needs clearing. Two calls whose GPU work
// overlaps in time (different streams, or different host threads on the same
// device) race on the array.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "host.h"
#include "illumina.h"
#include "kernels.h"

namespace {

// 64 Ki floats (256 KiB): enough for in_c * k * k up to 65536, e.g. 2621
// channels at k = 5 or 7281 at k = 3 (the network's widest layer is 704 x 5 x 5).
constexpr size_t kMaxPackedFloats = ILLUMINA_NOALLOC_DW_MAX_FLOATS;

__device__ __align__(256) float g_dw_packed[kMaxPackedFloats];

std::mutex g_mu;
std::vector<float *> g_addr;  // per device ordinal: device address of g_dw_packed

// Host code must not use g_dw_packed's name as a device address: resolve it
// once per device, with that device current.
float *packed_scratch_for_current_device(cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    throw illumina::Error(ILLUMINA_CUDA_ERROR, std::string("dwpw_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_mu);
  if ((size_t)dev >= g_addr.size()) g_addr.resize(dev + 1, nullptr);
  if (!g_addr[dev]) {
    // resolving the address is not a stream operation and may not be legal
    // while a capture is open: the first call on a device must come first
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess || cs != cudaStreamCaptureStatusNone)
      throw illumina::Error(ILLUMINA_INVALID_ARG,
                            "dwpw_noalloc: the first call on a device must precede stream capture (the stream is "
                            "being captured)");
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dw_packed);
    if (e != cudaSuccess || !p)
      throw illumina::Error(ILLUMINA_CUDA_ERROR,
                            std::string("dwpw_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_addr[dev] = static_cast<float *>(p);
  }
  return g_addr[dev];
}

void require(bool ok, const std::string &msg) {
  if (!ok) throw illumina::Error(ILLUMINA_INVALID_ARG, msg);
}

}  // namespace

extern "C" illumina_status illumina_op_dwpw_noalloc(const float *src, int in_h, int in_w, int in_c,
                                                    const float *dw_w, const float *dw_b, int mid_act,
                                                    const float *pw_w, const float *pw_b, int out_c, int k,
                                                    int stride, int act, const float *res, float *dst,
                                                    void *stream) {
  try {
    require(src && dw_w && dw_b && pw_w && pw_b && dst, "dwpw_noalloc: null pointer");
    require(in_c % 4 == 0 && out_c % 4 == 0 && in_c > 0 && out_c > 0,
            "dwpw_noalloc: channels must be multiples of 4");
    require(k == 3 || k == 5, "dwpw_noalloc: kernel size must be 3 or 5");
    require(stride == 1 || stride == 2, "dwpw_noalloc: stride must be 1 or 2");
    require(act >= 0 && act <= 3 && mid_act >= 0 && mid_act <= 3, "dwpw_noalloc: unknown activation");
    require((size_t)in_c * k * k <= kMaxPackedFloats,
            "dwpw_noalloc: in_c*k*k = " + std::to_string((size_t)in_c * k * k) + " exceeds the fixed scratch of " +
                std::to_string(kMaxPackedFloats) + " floats; use illumina_op_dwpw");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *packed = packed_scratch_for_current_device(st);
    cudaError_t e = illumina::gpu::pack_dw(dw_w, in_c, k, packed, 0, st);
    if (e != cudaSuccess) throw illumina::Error(ILLUMINA_CUDA_ERROR, std::string("dwpw_noalloc pack: ") + cudaGetErrorString(e));
    int pad = (k - 1) >> 1;
    illumina::gpu::GemmOp g;
    g.mode = 1, g.src = src, g.w = pw_w, g.bias = pw_b, g.res = res, g.dst = dst;
    g.H = in_h, g.W = in_w;
    g.OH = (in_h + 2 * pad - k) / stride + 1, g.OW = (in_w + 2 * pad - k) / stride + 1;
    g.M = (long)g.OH * g.OW, g.N = out_c, g.K = in_c;
    g.act = act, g.mid_act = mid_act, g.ks = k, g.stride = stride, g.dw_w = packed, g.dw_b = dw_b;
    e = illumina::gpu::gemm(illumina::gpu::F32, g, st);
    if (e != cudaSuccess) throw illumina::Error(ILLUMINA_CUDA_ERROR, std::string("dwpw_noalloc: ") + cudaGetErrorString(e));
    return ILLUMINA_OK;
  } catch (const illumina::Error &err) {
    illumina::set_last_error(err.what());
    return err.status;
  } catch (const std::exception &err) {
    illumina::set_last_error(err.what());
    return ILLUMINA_INVALID_ARG;
  }
}
