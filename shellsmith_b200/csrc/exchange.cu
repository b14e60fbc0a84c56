// K10 peer exchange of per-GPU attention partials over NVLink (config 4).
//
// Replaces the NCCL all-gather of the packed (out, lse) partial of a
// KV-sharded sequence (one [rows][D+1] fp32 block per GPU per attention
// layer, 16.4 KB at 16 heads x 256): the reference has no counterpart (it never
// shards a sequence). Every GPU maps every peer's receive buffer (CUDA IPC);
//   put  : one CTA per destination stores this GPU's block straight into that
//          peer's slot for this GPU (plain stores over NVLink, no multicast),
//          then publishes the layer's epoch in the peer's flag for this GPU
//          with a system-scope release store;
//   wait : one thread spins, with a bound, until every GPU's flag holds at
//          least the epoch (acquire loads), then the usual merge kernel reads
//          the blocks.
// Epochs grow by one per attention layer call (a device base the host stages
// per token plus the layer's offset), so a flag never needs resetting. The
// caller alternates two receive buffers by layer parity: a peer can be at most
// one layer ahead (its next put waits on this GPU's previous put through its
// own wait), so it never overwrites a block this GPU has not merged.
#include "common.cuh"
#include "peer.cuh"

namespace sc {
namespace {

// grid = world CTAs: CTA p copies `bytes` (a multiple of 16) from src to
// peer_dst[p], then sets *peer_flag[p] = epoch.
__global__ void __launch_bounds__(256)
    exchange_put_kernel(const uint4* __restrict__ src, int chunks, uint4* const* peer_dst,
                        unsigned int* const* peer_flag, const unsigned int* epoch_base,
                        unsigned int epoch_add) {
  pdl_wait();
  pdl_trigger();
  const int p = blockIdx.x;
  uint4* dst = peer_dst[p];
  for (int i = threadIdx.x; i < chunks; i += blockDim.x) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(peer_flag[p], *epoch_base + epoch_add);
  }
}

// One thread waits until flags[r] has reached the epoch for every r < world.
__global__ void exchange_wait_kernel(const unsigned int* flags, int world,
                                     const unsigned int* epoch_base, unsigned int epoch_add,
                                     uint32_t max_polls, unsigned int* status) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  wait_epochs(flags, world, *epoch_base + epoch_add, status, max_polls);
}

}  // namespace
}  // namespace sc

extern "C" int sc_exchange_put(const void* src, long long bytes, void* const* peer_dst,
                               unsigned int* const* peer_flag, const unsigned int* epoch_base,
                               unsigned int epoch_add, int world, void* stream) {
  using namespace sc;
  const char* name = "sc_exchange_put";
  SC_REQUIRE(src && peer_dst && peer_flag && epoch_base, SC_ERR_INVALID, "%s: null pointer",
             name);
  SC_REQUIRE(world > 0 && world <= 1024 && bytes > 0 && bytes % 16 == 0 &&
                 bytes / 16 < (1LL << 31),
             SC_ERR_INVALID, "%s: world=%d bytes=%lld (a positive multiple of 16)", name, world,
             bytes);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0, SC_ERR_INVALID,
             "%s: src must be 16-byte aligned", name);
  launch_pdl(exchange_put_kernel, dim3(world), dim3(256), 0, static_cast<cudaStream_t>(stream),
             static_cast<const uint4*>(src), (int)(bytes / 16),
             reinterpret_cast<uint4* const*>(peer_dst), peer_flag, epoch_base, epoch_add);
  return check_launch(name);
}

extern "C" int sc_exchange_wait_limited(const unsigned int* flags, int world,
                                        const unsigned int* epoch_base, unsigned int epoch_add,
                                        unsigned int max_polls, void* stream) {
  using namespace sc;
  const char* name = "sc_exchange_wait";
  SC_REQUIRE(flags && epoch_base, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(world > 0 && world <= 1024, SC_ERR_INVALID, "%s: world=%d", name, world);
  SC_REQUIRE(max_polls > 0, SC_ERR_INVALID, "%s: max_polls must be positive", name);
  launch_pdl(exchange_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
             flags, world, epoch_base, epoch_add, (uint32_t)max_polls, device_status_word());
  return check_launch(name);
}

extern "C" int sc_exchange_wait(const unsigned int* flags, int world,
                                const unsigned int* epoch_base, unsigned int epoch_add,
                                void* stream) {
  return sc_exchange_wait_limited(flags, world, epoch_base, epoch_add, sc::kPeerSpinLimit,
                                  stream);
}
