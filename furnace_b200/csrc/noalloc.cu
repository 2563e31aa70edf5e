// fz_dequant_dev_noalloc: quant::dequantize (src/quant.rs:261-281) on device
// buffers, allocating nothing.
//
// fz_dequant takes host buffers and allocates three device buffers per call
// (raw bytes, the repacked chunked layout, the f32 result); cudaFree
// synchronises the whole device.  A caller that converts GGUF tensors on the
// device while decode steps run on other streams -- a loader that fills the
// HBM left over after the weight pool and KV caches, or an inspection hook in
// a serving loop whose allocator owns all remaining device memory -- can
// neither stall the device nor count on a free allocation.  This variant
// takes device pointers and a stream, and keeps the repacked layout (the only
// scratch of the dequantization) in a fixed file-scope device array instead.
//
// Limits: the repacked tensor must fit in kScratchBytes (8 MiB); any tensor of
// at most 2 MiB of GGUF data does (the layout needs at most 3x the GGUF bytes,
// for block counts with no divisor between 2 and 8 / 64).  Larger requests
// are rejected with FZ_EINVAL before anything is launched.  The scratch is
// shared by every call on a device: two calls on the same device whose work
// overlaps in time (different streams, or different host threads) race on it.

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "fz_internal.h"
#include "kernels.h"

using namespace fz;

namespace {

constexpr size_t kScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

// The repacked (chunk-planar) copy of the tensor being dequantized.
static __device__ __align__(256) uint8_t g_dequant_scratch[kScratchBytes];

std::mutex g_mu;
uint8_t* g_scratch[kMaxDevices] = {};

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(FZ_ECUDA, "%s failed: %s", what, cudaGetErrorString(e));
}

// Address of the current device's copy of the scratch array, looked up once
// per device (with that device current).  The first call on a device does the
// lookup, which may load this module onto the device; make that first call
// before any stream capture begins.
uint8_t* scratch_for_current_device() {
  int dev = 0;
  ck(cudaGetDevice(&dev), "cudaGetDevice");
  need(dev >= 0 && dev < kMaxDevices, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[dev]) {
    void* p = nullptr;
    ck(cudaGetSymbolAddress(&p, g_dequant_scratch), "cudaGetSymbolAddress(dequant scratch)");
    g_scratch[dev] = static_cast<uint8_t*>(p);
  }
  return g_scratch[dev];
}

}  // namespace

extern "C" int fz_dequant_dev_noalloc(uint32_t dtype, const void* raw_dev, size_t nbytes, size_t n, float* out_dev,
                                      void* stream) {
  try {
    need(raw_dev && out_dev, "null argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t be, bb;
    need(block_geom(dtype, &be, &bb), "dequantization for type %u is not implemented", dtype);
    if (dtype == FZ_F32) {
      need(nbytes == n * 4, "F32 data is %zu bytes, expected %zu", nbytes, n * 4);
      if (n) ck(cudaMemcpyAsync(out_dev, raw_dev, n * 4, cudaMemcpyDeviceToDevice, s), "cudaMemcpyAsync");
      return FZ_OK;
    }
    need(is_quant(dtype), "dequantization for type %u is not implemented", dtype);
    need(n % be == 0, "element count %zu is not a multiple of %u", n, be);
    need(nbytes == n / be * bb, "data is %zu bytes, expected %zu (%zu blocks of %u)", nbytes, n / be * bb, n / be, bb);
    // the same view as fz_dequant: rows of k blocks, k the largest divisor of
    // the block count that keeps a row within one chunk of the device layout
    uint64_t nblk = n / be, kmax = be == 256 ? 8 : 64, k = 1;
    for (uint64_t t = kmax; t >= 1; t--)
      if (nblk % t == 0) {
        k = t;
        break;
      }
    // the scratch bound is checked on the 64-bit row count, before anything
    // is narrowed to the layout's 32-bit row index
    const uint64_t rows64 = nblk / k;
    const uint32_t cols = (uint32_t)(k * be);
    const uint64_t stride = dev_row_stride(dtype, cols);  // < 2^12: rows64 * stride cannot wrap below
    need(rows64 <= kScratchBytes, "fz_dequant_dev_noalloc: %zu blocks exceed the %zu-byte scratch", (size_t)nblk,
         kScratchBytes);
    const uint64_t lay_bytes = rows64 * stride;
    need(lay_bytes <= kScratchBytes,
         "fz_dequant_dev_noalloc: %zu blocks need %llu bytes of scratch, the limit is %zu (fz_dequant has none)",
         (size_t)nblk, (unsigned long long)lay_bytes, kScratchBytes);
    DevMat m;
    m.dtype = dtype;
    m.rows = (uint32_t)rows64;
    m.cols = cols;
    m.stride = stride;
    if (!m.rows) return FZ_OK;
    uint8_t* lay = scratch_for_current_device();
    // padding inside the layout starts at zero, as in fz_dequant's buffer
    ck(cudaMemsetAsync(lay, 0, lay_bytes, s), "cudaMemsetAsync");
    launch_repack(dtype, static_cast<const uint8_t*>(raw_dev), lay, 0, m.rows, m.rows, m.cols, s);
    m.ptr = lay;
    launch_dequant(m, 0, m.rows, out_dev, s);
    return FZ_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return FZ_EINVAL;
  }
}
