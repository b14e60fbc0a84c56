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
#include "common.cuh"

namespace sc {
namespace {

constexpr int kWarps = 4;

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
  static constexpr int U = (VPL >= 2) ? 4 : 8;               // passes in flight
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

template <typename ST>
int launch_gdn_decode(const char* name, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const float* g, const float* beta, ST* state, const int32_t* slot,
                      uint16_t* out, int B, int Hk, int Hv, int dk, int dv, int num_slots,
                      void* stream) {
  SC_REQUIRE(q && k && v && g && beta && state && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(B >= 0 && Hk > 0 && Hv > 0 && dv > 0, SC_ERR_INVALID,
             "%s: bad sizes B=%d Hk=%d Hv=%d dv=%d", name, B, Hk, Hv, dv);
  SC_REQUIRE(Hv % Hk == 0, SC_ERR_INVALID, "%s: Hv=%d not a multiple of Hk=%d", name, Hv, Hk);
  SC_REQUIRE(num_slots > 0 && (slot != nullptr || num_slots >= B), SC_ERR_INVALID,
             "%s: num_slots=%d for B=%d", name, num_slots, B);
  SC_REQUIRE((long long)B * Hv < (1LL << 31), SC_ERR_INVALID, "%s: B*Hv too large", name);
  if (B == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
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
}  // namespace sc

extern "C" int sc_gdn_decode(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v, const float* g,
                             const float* beta, float* state, const int32_t* state_slot,
                             sc_bf16* out, int B, int Hk, int Hv, int dk, int dv, int num_slots,
                             void* stream) {
  return sc::launch_gdn_decode<float>("sc_gdn_decode", q, k, v, g, beta, state, state_slot, out, B,
                                      Hk, Hv, dk, dv, num_slots, stream);
}

extern "C" int sc_gdn_decode_bf16(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                                  const float* g, const float* beta, sc_bf16* state,
                                  const int32_t* state_slot, sc_bf16* out, int B, int Hk, int Hv,
                                  int dk, int dv, int num_slots, void* stream) {
  return sc::launch_gdn_decode<uint16_t>("sc_gdn_decode_bf16", q, k, v, g, beta, state, state_slot,
                                         out, B, Hk, Hv, dk, dv, num_slots, stream);
}
