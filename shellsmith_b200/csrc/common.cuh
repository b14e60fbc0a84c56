// Shared helpers of the shellcache kernels: status reporting, bf16 packing,
// bounded mbarrier waits and the bulk-copy (TMA engine) primitives.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <utility>

#include "../../include/shellcache.h"

namespace sc {

// ---------------------------------------------------------------- host status
// The text of the last nonzero status on this host thread.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

#define SC_REQUIRE(cond, code, ...)                         \
  do {                                                      \
    if (!(cond)) return ::sc::set_error((code), __VA_ARGS__); \
  } while (0)

// ---------------------------------------------------------------- device status
// Bits of the device status word (sc_device_status reads and clears it).
enum : unsigned int {
  DEV_WAIT_TIMEOUT = 1u,    // a bounded mbarrier wait gave up
  DEV_BAD_INDEX = 2u,       // a page / slot index fell outside the pool
};
// Device address of the status word on the current device (host function;
// kernels receive it as an argument, so no relocatable device code is needed).
unsigned int* device_status_word();

__device__ __forceinline__ void flag_device(unsigned int* status, unsigned int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// Context length a split-K decode may attend for a sequence whose ctx_len entry
// is L: a negative length, or one whose pages exceed the block-table row
// (max_pages) or what the launch's splits cover (num_splits x pages_per_split),
// is flagged DEV_BAD_INDEX (by the CTA with `report` set) and clamped, so no
// read goes past the sequence's row of the block table and no page is dropped
// silently.
__device__ __forceinline__ int checked_ctx_len(int L, int page, int max_pages,
                                               int pages_per_split, int num_splits,
                                               unsigned int* status, bool report) {
  const long long cap_pages = min((long long)max_pages, (long long)num_splits * pages_per_split);
  const long long cap = cap_pages * page;
  if (L >= 0 && (long long)L <= cap) return L;
  if (report) flag_device(status, DEV_BAD_INDEX);
  return L < 0 ? 0 : (int)cap;
}

// ---------------------------------------------------------------- dependent launch
// Kernels of one decode step are launched as programmatic dependents of the
// kernel before them (launch_pdl): the next grid is scheduled while the
// current one runs, which hides the per-launch gap of a step made of many
// small kernels. A kernel launched that way calls pdl_wait() before it touches
// memory at all (every earlier kernel's writes are visible after it, and no
// earlier kernel still reads what it writes), then pdl_trigger(): the next
// grid launches once every CTA of this one has triggered or exited, so its
// CTAs only take resources this grid no longer needs. Both are no-ops in an
// ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- bf16 helpers
__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f(uint16_t x) { return __uint_as_float(uint32_t(x) << 16); }

__device__ __forceinline__ uint16_t f_to_bf16(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Packs (lo, hi) into one bf16x2 register, round-to-nearest-even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

// One try_wait on the given phase parity; true once that phase completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait: gives up after `limit` polls (each try_wait already blocks
// for a hardware-defined slice), flags DEV_WAIT_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned int* status,
                                                  uint32_t limit = (1u << 20)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  flag_device(status, DEV_WAIT_TIMEOUT);
  return false;
}

// Untiled bulk copy global -> shared (TMA engine), completion counted in bytes
// on `bar`. Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Untiled bulk copy shared -> global, tracked by the issuing thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// ---------------------------------------------------------------- warp MMA helpers
// ldmatrix x4 (optionally transposed) from a shared address.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col).
__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8 f32) += A(16x8 tf32, row) * B(8x8 tf32, col). Fragments (g = lane / 4,
// t = lane % 4): a0 (g, t), a1 (g + 8, t), a2 (g, t + 4), a3 (g + 8, t + 4);
// b0 (k = t, n = g), b1 (k = t + 4, n = g); d0/d1 (g, 2t / 2t + 1), d2/d3 (g + 8, ...).
__device__ __forceinline__ void mma_tf32_1688(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// x = big + small, both tf32 (round to nearest): big*big + big*small + small*big
// carries a product to about fp32 accuracy on the tf32 tensor path.
__device__ __forceinline__ void split_tf32(float x, uint32_t& big, uint32_t& small) {
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(big) : "f"(x));
  const float rest = x - __uint_as_float(big);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(small) : "f"(rest));
}

// acc (a 16x8 fp32 tile in the mma_tf32_1688 D layout) += A[16][K] * B[K][8], both
// fp32 in shared memory (row strides lda, ldb), as three tf32 products per k-step.
template <int K>
__device__ __forceinline__ void warp_gemm_tf32x3(float* acc, const float* A, int lda,
                                                 const float* B, int ldb, int lane) {
  const int g = lane >> 2, t = lane & 3;
  // Three accumulators, so the dependent MMA chain is K / 8 long, not 3K / 8.
  float c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 8) {
    uint32_t ab[4], as[4], bb[2], bs[2];
    split_tf32(A[g * lda + k0 + t], ab[0], as[0]);
    split_tf32(A[(g + 8) * lda + k0 + t], ab[1], as[1]);
    split_tf32(A[g * lda + k0 + t + 4], ab[2], as[2]);
    split_tf32(A[(g + 8) * lda + k0 + t + 4], ab[3], as[3]);
    split_tf32(B[(k0 + t) * ldb + g], bb[0], bs[0]);
    split_tf32(B[(k0 + t + 4) * ldb + g], bb[1], bs[1]);
    mma_tf32_1688(c1, as, bb);
    mma_tf32_1688(c2, ab, bs);
    mma_tf32_1688(acc, ab, bb);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) acc[e] += c1[e] + c2[e];
}

// Transposes one 8x8 b16 matrix held in the ldmatrix fragment layout.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

}  // namespace sc
