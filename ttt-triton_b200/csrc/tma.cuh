// Tensor-memory-accelerator (TMA) staging: 2-D tiled bulk tensor copies and 1-D bulk copies
// from global into shared memory, completed on an mbarrier, plus the host-side tensor maps.
//
// A 16 x 64 tile of 16-bit activations (one mini-batch of one stream, 128-byte rows) is
// copied with the 128-byte swizzle: inside each 1024-byte group of 8 rows the 16-byte chunk
// c of row r lands at chunk c ^ (r % 8), which is exactly the layout `swz128` addresses,
// so ldmatrix reads stay conflict-free. Destinations must be 1024-byte aligned for that.
//
// Waits are bounded in wall time: a thread that has polled an mbarrier for longer than
// kWaitLimitNs gives up, ORs its code into the device error word and reports failure, so
// a copy that never completes ends the kernel with an error instead of a hang.
#pragma once

#include <cuda.h>  // CUtensorMap and the cuTensorMapEncodeTiled types; the driver is not linked
#include <cuda_runtime.h>
#include <stdint.h>

namespace ttt {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s
constexpr unsigned int kDevErrTmaTimeout = 1u;                // bit in the device error word

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Makes mbarrier initialisation visible to the asynchronous (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 2-D tiled copy of the box at (x, y) of `map` into shared memory at dst.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 1-D bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of the mbarrier, at most limit_ns (kWaitLimitNs by default). On
// timeout ORs kDevErrTmaTimeout into *err (when given) and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int* err,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_test(bar, parity)) {
    if (global_ns() - t0 > limit_ns) {
      if (err) atomicOr(err, kDevErrTmaTimeout);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------- host
// Tensor map of a [rows][64] 16-bit matrix (row stride 128 bytes) read in box_rows x 64 boxes
// (box_rows <= 256) with the 128-byte swizzle. dtype_code: 1 bf16, 2 f16. Returns 0 or a
// TTT_ERR_* code.
int make_tile_map(CUtensorMap* map, const void* base, int dtype_code, unsigned long long rows, const char* who,
                  unsigned box_rows = 16);

// General 2-D tensor map over a row-major 16-bit matrix [rows][cols] (row stride in bytes, a
// multiple of 16) read in box_rows x box_cols boxes; swizzle128 selects the 128-byte swizzle
// (box_cols * 2 must then be 128).
int make_map_2d(CUtensorMap* map, const void* base, int dtype_code, unsigned long long cols, unsigned long long rows,
                unsigned long long row_stride_bytes, unsigned box_cols, unsigned box_rows, bool swizzle128,
                const char* who);

// Device address of the library's device error word on the current device.
int device_error_word(unsigned int** out, const char* who);

// Wait-expiry test switch (ttt_test_hold_first_stage): whether the tensor-core MLP forward
// holds back its first stage's copies, and the wait limit its launches use (ns).
bool test_hold_first_stage();
unsigned long long test_wait_limit_ns();

// Forward schedule switch (ttt_set_forward_schedule): whether the tensor-core MLP forward may
// use its balanced two-launch schedule, and the paired / alone mini-batch time ratio (x1000)
// it splits the sequence by.
bool forward_schedule_balanced();
int forward_paired_ratio_milli();

}  // namespace ttt
