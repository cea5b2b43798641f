// ABI-wide entry points: version, the per-thread last-error message and the device error
// word; host helpers shared by the kernels' entry points (TMA tensor maps).
#include <atomic>
#include <mutex>

#include "capi_common.cuh"
#include "common.cuh"
#include "tma.cuh"

extern "C" int ttt_abi_version(void) { return 10000; }

extern "C" const char* ttt_last_error(void) { return ttt::last_error_buffer(); }

namespace ttt {

// Bits set by kernels that gave up waiting (see tma.cuh); one word per device.
static __device__ unsigned int g_device_error;

int device_error_word(unsigned int** out, const char* who) {
  constexpr int kMaxDevices = 64;
  static unsigned int* addr[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(TTT_ERR_UNSUPPORTED, "%s: device %d out of range", who, dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_device_error);
    if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
    addr[dev] = static_cast<unsigned int*>(p);
  }
  *out = addr[dev];
  return TTT_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver the runtime already loaded (no link-time dependency).
static EncodeTiledFn encode_tiled(const char* who) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) fail(TTT_ERR_CUDA, "%s: cuTensorMapEncodeTiled is not available from the driver", who);
  return fn;
}

int make_map_2d(CUtensorMap* map, const void* base, int dtype_code, unsigned long long cols, unsigned long long rows,
                unsigned long long row_stride_bytes, unsigned box_cols, unsigned box_rows, bool swizzle128,
                const char* who) {
  EncodeTiledFn fn = encode_tiled(who);
  if (!fn) return TTT_ERR_CUDA;
  // A driver-API call uses the calling thread's current context, which a thread that has
  // made no runtime call yet (autograd's backward worker, say) does not have: bind the
  // current device's primary context first (no synchronisation).
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(TTT_ERR_CUDA, "%s: binding the device context: %s", who, cudaGetErrorString(e));
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype_code == DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TTT_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", who, (int)r);
  return TTT_OK;
}

int make_tile_map(CUtensorMap* map, const void* base, int dtype_code, unsigned long long rows, const char* who,
                  unsigned box_rows) {
  return make_map_2d(map, base, dtype_code, 64, rows, 128, 64, box_rows, true, who);
}

static std::atomic<int> g_test_hold{0};
static std::atomic<unsigned long long> g_test_wait_ns{kWaitLimitNs};

bool test_hold_first_stage() { return g_test_hold.load(std::memory_order_relaxed) != 0; }
unsigned long long test_wait_limit_ns() { return g_test_wait_ns.load(std::memory_order_relaxed); }

// Measured on B200 for the FF = 256 forward's two-stream CTAs: about 6.25 us per mini-batch
// for an engine whose CTA runs two streams, 4.17 us for one running alone; a sweep of the
// split over 1.40-1.65 at config 1 put the fastest forward at 1.55 (inference) and 1.50-1.55
// (with the training outputs).
constexpr int kPairedRatioMilli = 1550;
static std::atomic<int> g_fwd_balanced{1};
static std::atomic<int> g_fwd_ratio{kPairedRatioMilli};

bool forward_schedule_balanced() { return g_fwd_balanced.load(std::memory_order_relaxed) != 0; }
int forward_paired_ratio_milli() { return g_fwd_ratio.load(std::memory_order_relaxed); }

}  // namespace ttt

extern "C" unsigned long long ttt_kernel_launches(void) {
  return ttt::launch_counter().load(std::memory_order_relaxed);
}

extern "C" int ttt_set_forward_schedule(int balanced, int paired_ratio_milli) {
  TTT_REQUIRE(paired_ratio_milli == 0 || (paired_ratio_milli >= 1000 && paired_ratio_milli <= 4000), TTT_ERR_SHAPE,
              "ttt_set_forward_schedule: paired / alone ratio %d (x1000) outside [1000, 4000]", paired_ratio_milli);
  ttt::g_fwd_ratio.store(paired_ratio_milli ? paired_ratio_milli : ttt::kPairedRatioMilli);
  ttt::g_fwd_balanced.store(balanced ? 1 : 0);
  return ttt::ok();
}

extern "C" int ttt_test_hold_first_stage(int enable, unsigned long long wait_limit_ns) {
  TTT_REQUIRE(wait_limit_ns <= ttt::kWaitLimitNs, TTT_ERR_SHAPE,
              "ttt_test_hold_first_stage: wait limit %llu ns is above the library's %llu ns", wait_limit_ns,
              ttt::kWaitLimitNs);
  ttt::g_test_wait_ns.store(wait_limit_ns ? wait_limit_ns : ttt::kWaitLimitNs);
  ttt::g_test_hold.store(enable ? 1 : 0);
  return ttt::ok();
}

// Reads and clears the device error word of the current device (synchronises with it).
extern "C" int ttt_device_status(unsigned int* status) {
  TTT_REQUIRE(status, TTT_ERR_NULL, "ttt_device_status: NULL pointer argument");
  unsigned int* w = nullptr;
  int rc = ttt::device_error_word(&w, "ttt_device_status");
  if (rc) return rc;
  unsigned int v = 0;
  cudaError_t e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return ttt::fail(TTT_ERR_CUDA, "ttt_device_status: %s", cudaGetErrorString(e));
  if (v) {
    const unsigned int zero = 0;
    e = cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return ttt::fail(TTT_ERR_CUDA, "ttt_device_status: %s", cudaGetErrorString(e));
  }
  *status = v;
  return TTT_OK;
}
