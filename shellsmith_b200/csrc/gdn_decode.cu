// K1 gdn_decode: one-token gated-delta-net state update, state in place.
//
// Reference: studio_compute/numerics/gdn_token.py:18-79 (Metal kernel
// shellsmith_bf16_gdn_token_v1). Per (batch row b, value head h, value row i):
//   decayed = g * S[i,:];  delta = beta * (v[i] - decayed . k)
//   S[i,:]  = decayed + delta * k;  out[i] = S[i,:] . q
// Key head of h is h / (Hv / Hk) (gdn_token.py:57).
//
// B200 mapping. The state row S[i,:] (dk fp32) is the unit of work and the
// only large traffic: it is read once and written once. A warp covers a row
// with LPR lanes x VPL float4 (one 512-byte coalesced access for dk = 128),
// so the two dot products reduce with LPR-wide xor shuffles. Each warp issues
// U rows of loads before it computes, giving 16*U*VPL bytes in flight per
// lane. Loads and stores use the streaming (evict-first) cache hint: the
// state of one layer is far larger than L2 and is not reused in the step.
#include <type_traits>

#include "common.cuh"
#include "gdn_internal.cuh"

namespace sc {
namespace {

// Launch shape: warps per CTA and state rows each lane keeps in flight.
#ifndef SC_GDN_WARPS
#define SC_GDN_WARPS 4
#endif
#ifndef SC_GDN_ROWS_IN_FLIGHT
#define SC_GDN_ROWS_IN_FLIGHT 8
#endif
constexpr int kWarps = SC_GDN_WARPS;

template <typename ST>
struct StateIO;

template <>
struct StateIO<float> {
  static __device__ __forceinline__ float4 load(const float* p) {
    return __ldcs(reinterpret_cast<const float4*>(p));
  }
  static __device__ __forceinline__ void store(float* p, float4 x) {
    __stcs(reinterpret_cast<float4*>(p), x);
  }
  static __device__ __forceinline__ float round(float x) { return x; }
};

template <>
struct StateIO<uint16_t> {
  static __device__ __forceinline__ float4 load(const uint16_t* p) {
    uint2 r = __ldcs(reinterpret_cast<const uint2*>(p));
    return make_float4(bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y));
  }
  static __device__ __forceinline__ void store(uint16_t* p, float4 x) {
    uint2 r;
    r.x = pack_bf16x2(x.x, x.y);
    r.y = pack_bf16x2(x.z, x.w);
    __stcs(reinterpret_cast<uint2*>(p), r);
  }
  // The reference rounds the updated state to bf16 before the output dot.
  static __device__ __forceinline__ float round(float x) { return bf16_to_f(f_to_bf16(x)); }
};

__device__ __forceinline__ float4 load_bf16x4(const uint16_t* p) {
  uint2 r = *reinterpret_cast<const uint2*>(p);
  return make_float4(bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y));
}

template <int DK>
struct RowShape {
  static constexpr int LPR = (DK / 4 >= 32) ? 32 : DK / 4;  // lanes per state row
  static constexpr int VPL = DK / (4 * LPR);                 // float4 per lane per row
  static constexpr int RPP = 32 / LPR;                       // rows per warp pass
  static constexpr int U = (VPL >= 2) ? SC_GDN_ROWS_IN_FLIGHT / 2 : SC_GDN_ROWS_IN_FLIGHT;
  static constexpr int ROWS_PER_WARP = RPP * U;
  static constexpr int ROWS_PER_CTA = kWarps * ROWS_PER_WARP;
};

template <int DK, typename ST>
__global__ void __launch_bounds__(kWarps * 32)
    gdn_decode_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                      const uint16_t* __restrict__ v, const float* __restrict__ g,
                      const float* __restrict__ beta, ST* __restrict__ state,
                      const int32_t* __restrict__ state_slot, uint16_t* __restrict__ out,
                      int Hk, int Hv, int dv, int num_slots, unsigned int* status) {
  using Shape = RowShape<DK>;
  constexpr int LPR = Shape::LPR, VPL = Shape::VPL, RPP = Shape::RPP, U = Shape::U;

  const int bh = blockIdx.x;  // b * Hv + h
  const int b = bh / Hv;
  const int h = bh - b * Hv;
  const int slot = state_slot != nullptr ? state_slot[b] : b;
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0 && blockIdx.y == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const int kh = h / (Hv / Hk);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int sub = lane / LPR;
  const int l = lane - sub * LPR;
  const float decay = g[bh];
  const float bt = beta[bh];

  // This lane's slice of k and q: float4 chunks l, l + LPR, ...
  float4 kf[VPL], qf[VPL];
  const uint16_t* kp = k + ((size_t)b * Hk + kh) * DK;
  const uint16_t* qp = q + ((size_t)b * Hk + kh) * DK;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    kf[j] = load_bf16x4(kp + 4 * (j * LPR + l));
    qf[j] = load_bf16x4(qp + 4 * (j * LPR + l));
  }

  ST* S = state + ((size_t)slot * Hv + h) * (size_t)dv * DK;
  const int row0 = blockIdx.y * Shape::ROWS_PER_CTA + warp * Shape::ROWS_PER_WARP + sub;

  float4 s[U][VPL];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int row = row0 + u * RPP;
#pragma unroll
    for (int j = 0; j < VPL; ++j)
      s[u][j] = row < dv ? StateIO<ST>::load(S + (size_t)row * DK + 4 * (j * LPR + l))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
  }

#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int row = row0 + u * RPP;
    float pred = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      s[u][j].x *= decay;
      s[u][j].y *= decay;
      s[u][j].z *= decay;
      s[u][j].w *= decay;
      pred = fmaf(s[u][j].x, kf[j].x, pred);
      pred = fmaf(s[u][j].y, kf[j].y, pred);
      pred = fmaf(s[u][j].z, kf[j].z, pred);
      pred = fmaf(s[u][j].w, kf[j].w, pred);
    }
#pragma unroll
    for (int off = LPR / 2; off >= 1; off >>= 1) pred += __shfl_xor_sync(0xffffffffu, pred, off);
    const float vi = row < dv ? bf16_to_f(v[(size_t)bh * dv + row]) : 0.f;
    const float delta = bt * (vi - pred);
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      s[u][j].x = StateIO<ST>::round(fmaf(delta, kf[j].x, s[u][j].x));
      s[u][j].y = StateIO<ST>::round(fmaf(delta, kf[j].y, s[u][j].y));
      s[u][j].z = StateIO<ST>::round(fmaf(delta, kf[j].z, s[u][j].z));
      s[u][j].w = StateIO<ST>::round(fmaf(delta, kf[j].w, s[u][j].w));
      o = fmaf(s[u][j].x, qf[j].x, o);
      o = fmaf(s[u][j].y, qf[j].y, o);
      o = fmaf(s[u][j].z, qf[j].z, o);
      o = fmaf(s[u][j].w, qf[j].w, o);
    }
#pragma unroll
    for (int off = LPR / 2; off >= 1; off >>= 1) o += __shfl_xor_sync(0xffffffffu, o, off);
    if (row < dv) {
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        StateIO<ST>::store(S + (size_t)row * DK + 4 * (j * LPR + l), s[u][j]);
      if (l == 0) out[(size_t)bh * dv + row] = f_to_bf16(o);
    }
  }
}

// Fast path for an fp32 state with dk = 128: one CTA per (row b, value head h)
// streams the dv x 128 state through shared memory in 32-row chunks of 16 KiB,
// each one bulk copy (TMA engine) in and one bulk copy out, so an SM keeps
// ~3 x 64 KiB of state loads in flight without spending registers on them.
// Warp w updates rows 8w..8w+7 of each chunk in place in shared memory.
constexpr int kBulkRows = 32;
constexpr int kBulkChunkBytes = kBulkRows * 128 * 4;
#ifndef SC_GDN_BULK_CHUNKS
#define SC_GDN_BULK_CHUNKS 2  // 16 KiB chunks per CTA (32 KiB: ~7 CTAs per SM)
#endif
constexpr int kBulkChunksPerCta = SC_GDN_BULK_CHUNKS;

// NCH chunks of 32 rows per CTA: kBulkChunksPerCta for batches that fill the
// GPU, 1 (twice the CTAs) when a batch is too small to.
template <int NCH>
__global__ void __launch_bounds__(128)
    gdn_decode_bulk_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                           const uint16_t* __restrict__ v, const float* __restrict__ g,
                           const float* __restrict__ beta, float* __restrict__ state,
                           const int32_t* __restrict__ state_slot, uint16_t* __restrict__ out,
                           int Hk, int Hv, int dv, int num_slots, int wait_first,
                           unsigned int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int nchunks = NCH;
  // A dependent launch whose predecessor may write the state (or anything
  // else this kernel reads) waits before touching memory at all.
  if (wait_first) pdl_wait();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + nchunks * kBulkChunkBytes);
  const int chunk0 = blockIdx.y * nchunks;  // first 32-row chunk of this CTA
  const int bh = blockIdx.x;
  const int b = bh / Hv;
  const int h = bh - b * Hv;
  const int slot = state_slot != nullptr ? state_slot[b] : b;
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0 && blockIdx.y == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const int kh = h / (Hv / Hk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* S = state + ((size_t)slot * Hv + h) * (size_t)dv * 128 +
             (size_t)chunk0 * kBulkRows * 128;
  // One thread decides whether an earlier wait timed out, so the whole CTA
  // either streams its chunks or skips them.
  unsigned int* aborted = reinterpret_cast<unsigned int*>(bars + nchunks);

  if (tid == 0) {
    *aborted = status != nullptr &&
               (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT);
    for (int c = 0; c < nchunks; ++c) mbar_init(&bars[c], 1);
    fence_mbar_init();
    for (int c = 0; c < nchunks && !*aborted; ++c) {
      mbar_arrive_expect_tx(&bars[c], kBulkChunkBytes);
      bulk_g2s(smem + c * kBulkChunkBytes, S + (size_t)c * kBulkRows * 128, kBulkChunkBytes,
               &bars[c]);
    }
  }
  // Launched as a programmatic dependent of the kernel that makes q/k/v/g/beta,
  // the state loads above overlap that kernel; its outputs are read only after
  // this wait (a no-op in an ordinary launch).
  pdl_wait();
  pdl_trigger();
  const float4 kf = load_bf16x4(k + ((size_t)b * Hk + kh) * 128 + 4 * lane);
  const float4 qf = load_bf16x4(q + ((size_t)b * Hk + kh) * 128 + 4 * lane);
  const float decay = g[bh], bt = beta[bh];
  __syncthreads();  // barrier initialisation is visible before anyone waits
  if (*aborted) return;

  int ok = 1;
  for (int c = 0; c < nchunks; ++c) {
    if (ok && !mbar_wait_bounded(&bars[c], 0, status)) ok = 0;
    if (ok) {
      float4* rows = reinterpret_cast<float4*>(smem + c * kBulkChunkBytes);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int lr = 8 * warp + r;
        float4 s4 = rows[lr * 32 + lane];
        s4.x *= decay;
        s4.y *= decay;
        s4.z *= decay;
        s4.w *= decay;
        float pred = s4.x * kf.x + s4.y * kf.y + s4.z * kf.z + s4.w * kf.w;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) pred += __shfl_xor_sync(0xffffffffu, pred, off);
        const int row = (chunk0 + c) * kBulkRows + lr;
        const float delta = bt * (bf16_to_f(v[(size_t)bh * dv + row]) - pred);
        s4.x = fmaf(delta, kf.x, s4.x);
        s4.y = fmaf(delta, kf.y, s4.y);
        s4.z = fmaf(delta, kf.z, s4.z);
        s4.w = fmaf(delta, kf.w, s4.w);
        float o = s4.x * qf.x + s4.y * qf.y + s4.z * qf.z + s4.w * qf.w;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) o += __shfl_xor_sync(0xffffffffu, o, off);
        rows[lr * 32 + lane] = s4;
        if (lane == 0) out[(size_t)bh * dv + row] = f_to_bf16(o);
      }
    }
    fence_proxy_async_smem();  // this thread's smem writes are visible to the bulk store
    __syncthreads();
    if (tid == 0 && ok) {
      bulk_s2g(S + (size_t)c * kBulkRows * 128, smem + c * kBulkChunkBytes, kBulkChunkBytes);
      bulk_commit();
    }
  }
  if (tid == 0) {
    if (!ok) {
      // A load never arrived (flagged): let the copies still in flight land
      // before the CTA's shared memory is released.
      for (int c = 0; c < nchunks; ++c) mbar_wait_bounded(&bars[c], 0, status);
    }
    bulk_wait_read_all();
  }
}

template <typename ST>
int launch_gdn_decode(const char* name, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const float* g, const float* beta, ST* state, const int32_t* slot,
                      uint16_t* out, int B, int Hk, int Hv, int dk, int dv, int num_slots,
                      void* stream, BulkLaunch mode = BulkLaunch::kDependent) {
  SC_REQUIRE(q && k && v && g && beta && state && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(B >= 0 && Hk > 0 && Hv > 0 && dv > 0, SC_ERR_INVALID,
             "%s: bad sizes B=%d Hk=%d Hv=%d dv=%d", name, B, Hk, Hv, dv);
  SC_REQUIRE(Hv % Hk == 0, SC_ERR_INVALID, "%s: Hv=%d not a multiple of Hk=%d", name, Hv, Hk);
  SC_REQUIRE(num_slots > 0 && (slot != nullptr || num_slots >= B), SC_ERR_INVALID,
             "%s: num_slots=%d for B=%d", name, num_slots, B);
  SC_REQUIRE((long long)B * Hv < (1LL << 31), SC_ERR_INVALID, "%s: B*Hv too large", name);
  if (B == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if constexpr (std::is_same<ST, float>::value) {
    if (gdn_bulk_supported(dk, dv))
      return gdn_bulk_launch(name, q, k, v, g, beta, state, slot, out, B, Hk, Hv, dv, num_slots,
                             s, mode);
  }
  dim3 block(kWarps * 32);
#define SC_GDN_CASE(DK_)                                                                     \
  case DK_: {                                                                                \
    dim3 grid(B * Hv, (dv + RowShape<DK_>::ROWS_PER_CTA - 1) / RowShape<DK_>::ROWS_PER_CTA); \
    gdn_decode_kernel<DK_, ST><<<grid, block, 0, s>>>(q, k, v, g, beta, state, slot, out, Hk, \
                                                      Hv, dv, num_slots,                     \
                                                      device_status_word());                 \
    break;                                                                                   \
  }
  switch (dk) {
    SC_GDN_CASE(32)
    SC_GDN_CASE(64)
    SC_GDN_CASE(128)
    SC_GDN_CASE(256)
    default:
      return set_error(SC_ERR_UNSUPPORTED, "%s: dk=%d not in {32,64,128,256}", name, dk);
  }
#undef SC_GDN_CASE
  return check_launch(name);
}

}  // namespace

bool gdn_bulk_supported(int dk, int dv) {
  return dk == 128 && dv % (kBulkRows * kBulkChunksPerCta) == 0;
}

int gdn_bulk_launch(const char* name, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                    const float* g, const float* beta, float* state, const int32_t* slot,
                    uint16_t* out, int B, int Hk, int Hv, int dv, int num_slots, cudaStream_t s,
                    BulkLaunch mode) {
  static int configured[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(SC_ERR_CUDA, "%s: device %d", name, dev);
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(gdn_decode_bulk_kernel<kBulkChunksPerCta>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kBulkChunksPerCta * (kBulkChunkBytes + 8) + 8);
    if (err == cudaSuccess)
      err = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess)
      return set_error(SC_ERR_CUDA, "%s: setup: %s", name, cudaGetErrorString(err));
    configured[dev] = 1;
  }
  // Up to ~48 two-chunk CTAs per SM (at 32 value heads, fewer than ~110 rows): one
  // 16 KiB chunk per CTA instead, twice the CTAs and more loads in flight. Measured on
  // config-3 steps: 64 rows 3.72 -> 3.62 ms, 32 rows 2.30 -> 2.20 ms, 128 rows even,
  // 256 rows 12.49 -> 12.68 ms.
  const bool small =
      (long long)B * Hv * (dv / (kBulkRows * kBulkChunksPerCta)) < 48LL * sms[dev];
  const int nch = small ? 1 : kBulkChunksPerCta;
  const int smem = nch * (kBulkChunkBytes + 8) + 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B * Hv, dv / (kBulkRows * nch));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = mode == BulkLaunch::kOrdinary ? 0 : 1;
  const int wait_first = mode == BulkLaunch::kDependent ? 1 : 0;
  cudaError_t err =
      small ? cudaLaunchKernelEx(&cfg, gdn_decode_bulk_kernel<1>, q, k, v, g, beta, state, slot,
                                 out, Hk, Hv, dv, num_slots, wait_first, device_status_word())
            : cudaLaunchKernelEx(&cfg, gdn_decode_bulk_kernel<kBulkChunksPerCta>, q, k, v, g,
                                 beta, state, slot, out, Hk, Hv, dv, num_slots, wait_first,
                                 device_status_word());
  if (err != cudaSuccess)
    return set_error(SC_ERR_CUDA, "%s: launch: %s", name, cudaGetErrorString(err));
  return check_launch(name);
}

}  // namespace sc

extern "C" int sc_gdn_decode(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v, const float* g,
                             const float* beta, float* state, const int32_t* state_slot,
                             sc_bf16* out, int B, int Hk, int Hv, int dk, int dv, int num_slots,
                             void* stream) {
  return sc::launch_gdn_decode<float>("sc_gdn_decode", q, k, v, g, beta, state, state_slot, out, B,
                                      Hk, Hv, dk, dv, num_slots, stream);
}

extern "C" int sc_gdn_decode_chained(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                                     const float* g, const float* beta, float* state,
                                     const int32_t* state_slot, sc_bf16* out, int B, int Hk,
                                     int Hv, int dk, int dv, int num_slots, void* stream) {
  return sc::launch_gdn_decode<float>("sc_gdn_decode_chained", q, k, v, g, beta, state,
                                      state_slot, out, B, Hk, Hv, dk, dv, num_slots, stream,
                                      sc::BulkLaunch::kStateAhead);
}

extern "C" int sc_gdn_decode_bf16(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                                  const float* g, const float* beta, sc_bf16* state,
                                  const int32_t* state_slot, sc_bf16* out, int B, int Hk, int Hv,
                                  int dk, int dv, int num_slots, void* stream) {
  return sc::launch_gdn_decode<uint16_t>("sc_gdn_decode_bf16", q, k, v, g, beta, state, state_slot,
                                         out, B, Hk, Hv, dk, dv, num_slots, stream);
}
