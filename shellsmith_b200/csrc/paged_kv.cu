// K4 paged KV append, its inverse (gather) and the page copy of a fork.
//
// Reference: the KV write of studio_compute/mlx_request_cache.py:59-63
// (OwnedKV.update_and_fetch concatenates the new token along L) and mlx-vlm's
// KVCache.update_and_fetch. Here the cache is a page pool and a token's slot
// (page * P + offset) comes from the host block manager.
//
// Pool layout: kv_pool[num_pages][Hkv][2][P][D] bf16. The row of token t in a
// (page, head, K|V) block keeps its 16-byte chunk c at position c ^ (t & 7):
// one bulk copy of the block is then bank-conflict-free for ldmatrix.
//
// Each thread moves one 16-byte chunk; a warp writes whole 512-byte rows for
// D = 256, so the scatter is coalesced per row.
#include "common.cuh"

namespace sc {
namespace {

__device__ __forceinline__ size_t pool_row(int64_t page, int kvh, int which, int off, int Hkv,
                                           int P, int D) {
  return ((((size_t)page * Hkv + kvh) * 2 + which) * P + off) * (size_t)D;
}

__global__ void kv_append_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v,
                                 uint16_t* __restrict__ pool, const int64_t* __restrict__ slots,
                                 long long total, int Hkv, int D, int P, int64_t num_pages,
                                 unsigned int* status) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int chunks = D / 8;
  const int c = (int)(idx % chunks);
  long long r = idx / chunks;
  const int which = (int)(r % 2);
  r /= 2;
  const int kvh = (int)(r % Hkv);
  const long long tok = r / Hkv;
  const int64_t slot = slots[tok];
  if (slot < 0) return;
  const int64_t page = slot / P;
  const int off = (int)(slot - page * P);
  if (page >= num_pages) {
    flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const uint4* src = (which ? v : k) + ((size_t)tok * Hkv + kvh) * chunks + c;
  uint16_t* dst = pool + pool_row(page, kvh, which, off, Hkv, P, D) + 8 * (c ^ (off & 7));
  *reinterpret_cast<uint4*>(dst) = *src;
}

__global__ void kv_gather_kernel(const uint16_t* __restrict__ pool, const int64_t* __restrict__ slots,
                                 uint4* __restrict__ k_out, uint4* __restrict__ v_out,
                                 long long total, int Hkv, int D, int P, int64_t num_pages,
                                 unsigned int* status) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int chunks = D / 8;
  const int c = (int)(idx % chunks);
  long long r = idx / chunks;
  const int which = (int)(r % 2);
  r /= 2;
  const int kvh = (int)(r % Hkv);
  const long long tok = r / Hkv;
  uint4* dst = (which ? v_out : k_out) + ((size_t)tok * Hkv + kvh) * chunks + c;
  const int64_t slot = slots[tok];
  const int64_t page = slot / P;
  if (slot < 0 || page >= num_pages) {
    if (slot >= 0) flag_device(status, DEV_BAD_INDEX);
    *dst = make_uint4(0, 0, 0, 0);
    return;
  }
  const int off = (int)(slot - page * P);
  *dst = *reinterpret_cast<const uint4*>(pool + pool_row(page, kvh, which, off, Hkv, P, D) +
                                         8 * (c ^ (off & 7)));
}

__global__ void kv_copy_pages_kernel(uint4* __restrict__ pool, const int32_t* __restrict__ src,
                                     const int32_t* __restrict__ dst, long long total,
                                     int page_chunks, int64_t num_pages, unsigned int* status) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const long long i = idx / page_chunks;
  const int c = (int)(idx - i * page_chunks);
  const int32_t s = src[i], d = dst[i];
  if (s < 0 || d < 0 || s >= num_pages || d >= num_pages) {
    flag_device(status, DEV_BAD_INDEX);
    return;
  }
  pool[(size_t)d * page_chunks + c] = pool[(size_t)s * page_chunks + c];
}

int check_pool_args(const char* name, int Hkv, int D, int P, int64_t num_pages) {
  SC_REQUIRE(Hkv > 0 && num_pages > 0, SC_ERR_INVALID, "%s: bad Hkv=%d num_pages=%lld", name, Hkv,
             (long long)num_pages);
  SC_REQUIRE(D == 64 || D == 128 || D == 256, SC_ERR_UNSUPPORTED, "%s: D=%d not in {64,128,256}",
             name, D);
  SC_REQUIRE(P == 8 || P == 16 || P == 32, SC_ERR_UNSUPPORTED, "%s: P=%d not in {8,16,32}", name,
             P);
  return SC_OK;
}

}  // namespace
}  // namespace sc

extern "C" int sc_kv_append(const sc_bf16* k, const sc_bf16* v, sc_bf16* kv_pool,
                            const int64_t* slot_mapping, int ntok, int Hkv, int D, int P,
                            int64_t num_pages, void* stream) {
  const char* name = "sc_kv_append";
  if (int rc = sc::check_pool_args(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(k && v && kv_pool && slot_mapping, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(ntok >= 0, SC_ERR_INVALID, "%s: ntok=%d", name, ntok);
  if (ntok == 0) return SC_OK;
  const long long total = (long long)ntok * Hkv * 2 * (D / 8);
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  cudaError_t err = sc::launch_pdl(
      sc::kv_append_kernel, dim3((unsigned)blocks), dim3(threads), 0,
      static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(k),
      reinterpret_cast<const uint4*>(v), reinterpret_cast<uint16_t*>(kv_pool), slot_mapping,
      total, Hkv, D, P, num_pages, sc::device_status_word());
  if (err != cudaSuccess)
    return sc::set_error(SC_ERR_CUDA, "%s: launch: %s", name, cudaGetErrorString(err));
  return sc::check_launch(name);
}

extern "C" int sc_kv_gather(const sc_bf16* kv_pool, const int64_t* slot_mapping, sc_bf16* k_out,
                            sc_bf16* v_out, int ntok, int Hkv, int D, int P, int64_t num_pages,
                            void* stream) {
  const char* name = "sc_kv_gather";
  if (int rc = sc::check_pool_args(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(kv_pool && slot_mapping && k_out && v_out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(ntok >= 0, SC_ERR_INVALID, "%s: ntok=%d", name, ntok);
  if (ntok == 0) return SC_OK;
  const long long total = (long long)ntok * Hkv * 2 * (D / 8);
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  sc::kv_gather_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      kv_pool, slot_mapping, reinterpret_cast<uint4*>(k_out), reinterpret_cast<uint4*>(v_out),
      total, Hkv, D, P, num_pages, sc::device_status_word());
  return sc::check_launch(name);
}

extern "C" int sc_kv_copy_pages(sc_bf16* kv_pool, const int32_t* src, const int32_t* dst,
                                int npages, int Hkv, int D, int P, int64_t num_pages,
                                void* stream) {
  const char* name = "sc_kv_copy_pages";
  if (int rc = sc::check_pool_args(name, Hkv, D, P, num_pages)) return rc;
  SC_REQUIRE(kv_pool && src && dst, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(npages >= 0, SC_ERR_INVALID, "%s: npages=%d", name, npages);
  if (npages == 0) return SC_OK;
  const int page_chunks = Hkv * 2 * P * D / 8;
  const long long total = (long long)npages * page_chunks;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  sc::kv_copy_pages_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint4*>(kv_pool), src, dst, total, page_chunks, num_pages,
      sc::device_status_word());
  return sc::check_launch(name);
}
