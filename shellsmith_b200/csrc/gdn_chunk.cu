// K2+K3 gdn_chunk_prefill: chunk-64 gated-delta prefill on tcgen05 tensor cores.
//
// Reference: studio_compute/numerics/ops.py:151-215 `gated_delta_chunked`
// (WY/UT chunk form, _invert_unit_lower :54-85, _scan_forward :88-104) and the
// fused Metal path numerics/gdn_fused.py:86-171. Per chunk of C = 64 tokens,
// with lg = cumsum(log clamp(g, 1e-6, 1)), decay = e^lg, R_tj = e^(lg_t - lg_j),
// r_t = e^(lg_63 - lg_t), A_tj = beta_t R_tj (k_t . k_j) (j < t), X = (I + A)^-1,
// m_tj = R_tj (q_t . k_j) (j <= t), the reference computes u0 = X(beta v),
// kt = X(beta decay k), q_eff = decay q - m kt, mu0 = m u0 and scans
//   O = mu0 + q_eff S^T,  U = u0 - kt S^T,  S <- decay_63 S + (r U)^T K.
// Substituting gives the same numbers with two fewer products:
//   W = beta (V - decay (K S^T)),  U = X W,  O = decay (Q S^T) + (m X) W,
//   S <- decay_63 S + (r U)^T K.
//
// B200 mapping. One CTA owns one (sequence, value head) and walks its chunks in
// order; the 128 x 128 fp32 state lives in tensor memory the whole time. Twelve
// warps in two groups: warps 0-7 run chunk c's state chain (X split, Y, G12, W,
// G34, U r, GS, the O rows) while warps 8-11 prepare chunk c + 1 (gates, G0,
// A / m, the inverse); mbarriers carry the hand-offs both ways. Everything is
// computed transposed, so TMEM lane = value row i:
//   G0  [K;Q] K^T            -> A (fp32 smem), m        M128 N64  K128
//   Y   m X                  -> rows 64.. of [X;Y]      M128 N64  K64   A in TMEM
//   G12 S [K;Q]^T            -> P1^T | P2^T             M128 N128 K128  A in TMEM
//   G34 W^T [X;Y]^T (+= 0 | decay P2^T) -> U^T | O^T    M128 N128 K64   A in TMEM
//   GS  (U^T r) K  (+= decay_63 S)                      M128 N128 K64   A in TMEM
// The A operands in TMEM (m, S, W^T, (U^T r), as bf16 hi/lo pair columns) are
// written by the threads that own their lanes; B operands come from shared memory.
// Q/K/V chunk tiles arrive by TMA (128-byte swizzle, no multicast); the
// unit-lower inverse solves its 8 x 8 diagonal blocks column-per-thread in fp32
// and builds the off-diagonal blocks from them (warp mma.sync tf32 tiles, each
// product as three tf32 products, fp32-accurate). Operands that feed the
// fp32 state (S, W, X, Y, U) are split into bf16 hi + lo and multiplied as
// hi*hi + hi*lo + lo*hi, which keeps the state within ~1e-5 of fp32 math.
#include <cudaTypedefs.h>
#include <math_constants.h>

#include <mutex>

#include "tc.cuh"

namespace sc {
namespace {

constexpr int kC = 64;    // chunk length
constexpr int kD = 128;   // key and value width
// Warps 0-7 run the state chain of chunk c (two per TMEM lane quarter, `hf` picks
// the column half); warps 8-11 prepare chunk c + 1 meanwhile (one per quarter).
constexpr int kMainThreads = 256;
constexpr int kPrepThreads = 128;
constexpr int kThreads = kMainThreads + kPrepThreads;
constexpr int kMainBar = 1, kPrepBar = 2;  // named barriers of the two groups
constexpr int kKQBufs = 3;  // K/Q tiles of chunk c live from the prep's G0 to the chain's GS

// Shared memory plan (byte offsets from a 1024-aligned base). The MMA operands
// that are built per TMEM lane (S, W, U r and m as bf16 hi/lo) stay in tensor
// memory; shared memory holds the TMA tiles, the B operands built from X and Y,
// and the fp32 scratch of the inverse.
constexpr uint32_t OFF_KQ = 0;          // kKQBufs x [2 dk halves][K rows 0-63 | Q rows 64-127][128 B]
constexpr uint32_t KQ_BYTES = 32768;
constexpr uint32_t OFF_V = kKQBufs * KQ_BYTES;  // [2 dv halves][64 rows][128 B]
constexpr uint32_t OFF_XYH = OFF_V + 16384;     // [X rows 0-63 | Y rows 64-127][128 B] hi
constexpr uint32_t OFF_XYL = OFF_XYH + 16384;   // lo
constexpr uint32_t OFF_XTH = OFF_XYL + 16384;   // X^T rows hi [64 rows][128 B]
constexpr uint32_t OFF_XTL = OFF_XTH + 8192;         // lo
constexpr uint32_t OFF_AMAT = OFF_XTL + 8192;   // A (strict lower) fp32 [64][kAStride], then X
constexpr int kAStride = 68;            // fp32 row stride of A (conflict-free float4 rows)
constexpr uint32_t OFF_TBUF = OFF_AMAT + 64 * kAStride * 4;  // inverse scratch [32][kTStride]
constexpr int kTStride = 40;            // fp32 row stride of the inverse scratch
constexpr uint32_t OFF_SMALL = OFF_TBUF + 32 * kTStride * 4;  // kGateSets gate sets
                                        // [lg, beta, decay, r, inv][64] floats; barriers; TMEM base
constexpr int kMaxRankedSeqs = 4096;    // longer varlen batches keep their order
// The varlen ranking stages cu_seqlens in the A scratch before the first chunk.
static_assert((kMaxRankedSeqs + 2) * 4 <= 64 * kAStride * 4, "ranking scratch exceeds A");
static_assert(OFF_V % 1024 == 0 && OFF_XYH % 1024 == 0 && OFF_XYL % 1024 == 0 &&
                  OFF_XTH % 1024 == 0 &&
                  OFF_XTL % 1024 == 0,
              "swizzled tiles need 1024-byte alignment");
constexpr int kGateSet = 5 * 64;  // floats of one chunk's gate arrays
constexpr int kGateSets = 3;      // chunk c uses set c % 3 (made a chunk ahead by the prep)
constexpr uint32_t SMEM_BYTES = OFF_SMALL + kGateSets * kGateSet * 4 + 128 + 1024;  // + slack
static_assert(SMEM_BYTES <= 232448, "shared memory plan exceeds 227 KB");
// Each CTA allocates all 512 TMEM columns, so two must never share an SM: the
// shared memory plan alone keeps a second one off (228 KB per SM).
static_assert(2 * SMEM_BYTES > 228 * 1024, "a second CTA per SM would wait for TMEM");

// 32 fp32 values of this thread's TMEM lane as bf16 hi + lo pair columns: 16
// columns at hi_col and 16 at lo_col (an A operand of a K = 32 slice).
__device__ __forceinline__ void tmem_store_hilo(uint32_t hi_col, uint32_t lo_col,
                                                const float* x) {
  uint32_t hi[16], lo[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    hi[e] = pack_bf16x2(x[2 * e], x[2 * e + 1]);
    lo[e] = pack_bf16x2(x[2 * e] - bf16_lo(hi[e]), x[2 * e + 1] - bf16_hi(hi[e]));
  }
  tc::tmem_st16(hi_col, hi);
  tc::tmem_st16(lo_col, lo);
}

// TMEM columns (512 allocated).
// The state; P1 | P2 and then U | O (and Y before G12); KK^T | QK^T (the prep);
// m hi | lo (the prep, read by Y); S, then W^T, then (U^T r) as bf16 hi / lo pairs.
constexpr uint32_t T_S = 0, T_P = 128, T_KK = 256, T_M = 320;
constexpr uint32_t T_SH = 384, T_SL = 448;

__device__ __forceinline__ void store_chunks_hilo(uint8_t* hi, uint8_t* lo, int row, int c0,
                                                  const float* x) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = x[8 * c + 2 * e], b = x[8 * c + 2 * e + 1];
      h[e] = pack_bf16x2(a, b);
      l[e] = pack_bf16x2(a - bf16_lo(h[e]), b - bf16_hi(h[e]));
    }
    const uint32_t off = (uint32_t)row * 128u + (uint32_t)((((c0 + c) ^ (row & 7)) << 4));
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// Stores 8 consecutive values as one 16-byte chunk (chunk index c of a row) of
// a hi tile and a lo tile.
__device__ __forceinline__ void store_chunk8_hilo(uint8_t* hi, uint8_t* lo, int row, int c,
                                                  const float* x) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = x[2 * e], b = x[2 * e + 1];
    h[e] = pack_bf16x2(a, b);
    l[e] = pack_bf16x2(a - bf16_lo(h[e]), b - bf16_hi(h[e]));
  }
  const uint32_t off = (uint32_t)row * 128u + (uint32_t)(((c ^ (row & 7)) << 4));
  *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Named barrier of one warp group that also ANDs `pred` over the group's threads.
__device__ __forceinline__ int group_sync_and(int id, int nthreads, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred), "r"(id), "r"(nthreads)
      : "memory");
  return r;
}
__device__ __forceinline__ void group_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn_chunk_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ g,
                     const float* __restrict__ beta, float* __restrict__ state,
                     const int32_t* __restrict__ state_slot,
                     const int32_t* __restrict__ cu_seqlens, uint16_t* __restrict__ out, int Hk,
                     int Hv, int T_fixed, int num_slots, unsigned int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  // Gate arrays of a chunk (set c % kGateSets): log2 prefix sums lg, beta, decay =
  // 2^lg, r = 2^(lg_63 - lg), inv = 2^(lg_0 - lg) (the column factor of the decay
  // ratios).
  float* gate_sets = reinterpret_cast<float*>(sm + OFF_SMALL);
  uint64_t* bar_kq = reinterpret_cast<uint64_t*>(gate_sets + kGateSets * kGateSet);  // [kKQBufs]
  uint64_t* bar_v = bar_kq + kKQBufs;   // V tile
  uint64_t* bar_mma = bar_v + 1;        // the state chain's MMAs
  uint64_t* bar_g0 = bar_mma + 1;       // the prep's G0
  uint64_t* bar_mfree = bar_g0 + 1;     // a chunk's X split and Y have read X, m and X^T
  uint64_t* bar_full = bar_mfree + 1;   // [2]: a chunk's prep is in place
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar_full + 2);
  float* Xf = reinterpret_cast<float*>(sm + OFF_AMAT);  // A, inverted in place into X
  float* Tbuf = reinterpret_cast<float*>(sm + OFF_TBUF);

  const int bh = blockIdx.x;
  int b = bh / Hv;
  const int h = bh - b * Hv;
  const int kh = h / (Hv / Hk);
  // Varlen batches run longest sequence first: when the grid is more than one
  // wave, the CTAs left for the second wave belong to the shortest sequences.
  // Block row b takes the sequence of rank b (length descending, index
  // ascending), ranked here from cu_seqlens staged in the A scratch, which the
  // chunk loop first writes long after.
  if (cu_seqlens != nullptr && (int)(gridDim.x / Hv) <= kMaxRankedSeqs) {
    const int nseq = (int)(gridDim.x / Hv);
    int* s_cu = reinterpret_cast<int*>(sm + OFF_AMAT);
    for (int i = threadIdx.x; i <= nseq; i += blockDim.x) s_cu[i] = cu_seqlens[i];
    __syncthreads();
    for (int i = threadIdx.x; i < nseq; i += blockDim.x) {
      const int li = s_cu[i + 1] - s_cu[i];
      int rank = 0;
      for (int j = 0; j < nseq; ++j) {
        const int lj = s_cu[j + 1] - s_cu[j];
        rank += (lj > li || (lj == li && j < i)) ? 1 : 0;
      }
      if (rank == b) s_cu[nseq + 1] = i;
    }
    __syncthreads();
    b = s_cu[nseq + 1];
  }
  const int start = cu_seqlens != nullptr ? cu_seqlens[b] : b * T_fixed;
  const int len = cu_seqlens != nullptr ? cu_seqlens[b + 1] - start : T_fixed;
  const int slot = state_slot != nullptr ? state_slot[b] : b;
  if (slot < 0 || len <= 0) return;  // uniform over the CTA
  if (slot >= num_slots) {
    if (threadIdx.x == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  // After any bounded wait has given up on this device, later CTAs stop at once.
  if (status != nullptr && (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT))
    return;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane_id = tid & 31;
  const bool is_prep = warp >= kMainThreads / 32;
  const int quarter = warp & 3;
  const int hf = (warp >> 2) & 1;  // the state chain's column half
  const int row = quarter * 32 + lane_id;  // TMEM lane: value row i (or token row t)
  const uint32_t lane = (uint32_t)(quarter * 32) << 16;

  if (tid == 0) {
    for (int i = 0; i < kKQBufs; ++i) mbar_init(&bar_kq[i], 1);
    mbar_init(bar_v, 1);
    mbar_init(bar_mma, 1);
    mbar_init(bar_g0, 1);
    mbar_init(bar_mfree, 2);  // the chain's arrival after the X split, and Y's commit
    mbar_init(&bar_full[0], 1);
    mbar_init(&bar_full[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(s_tmem, 512);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  const int nchunks = (len + kC - 1) / kC;

  auto issue_kq = [&](int chunk) {  // one thread
    const int bi = chunk % kKQBufs;
    uint8_t* buf = sm + OFF_KQ + bi * KQ_BYTES;
    const int t0 = start + chunk * kC;
    mbar_arrive_expect_tx(&bar_kq[bi], 4 * 8192);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      tc::tma_load_3d(buf + half * 16384, &tm_k, half * 64, kh, t0, &bar_kq[bi]);
      tc::tma_load_3d(buf + half * 16384 + 8192, &tm_q, half * 64, kh, t0, &bar_kq[bi]);
    }
  };
  auto issue_v = [&](int chunk) {  // one thread
    const int t0 = start + chunk * kC;
    mbar_arrive_expect_tx(bar_v, 2 * 8192);
#pragma unroll
    for (int half = 0; half < 2; ++half)
      tc::tma_load_3d(sm + OFF_V + half * 8192, &tm_v, half * 64, h, t0, bar_v);
  };

  int ok = 1;
  float* srow = state + ((size_t)slot * Hv + h) * kD * kD + (size_t)row * kD + 64 * hf;
  if (is_prep) {
    // ================= the prep of chunk n (warps 8-11): gates, G0, A / m, the
    // inverse and the X splits, one chunk ahead of the state chain.
    const int ptid = tid - kMainThreads;
    const int pw = quarter;  // this warp's TMEM lane quarter
    uint32_t g0_phase = 0;
    int g0_pending = 0;
    // Warp 8 reads a chunk's g and beta (tokens 2 lane, 2 lane + 1) a chunk
    // before it makes that chunk's gate set.
    float gn0 = 1.f, gn1 = 1.f, bn0 = 0.f, bn1 = 0.f;
    auto fetch_gates = [&](int chunk) {
      const int n = min(kC, len - chunk * kC);
      const int t0 = 2 * lane_id;
      const size_t at = (size_t)(start + chunk * kC + t0) * Hv + h;
      gn0 = t0 < n ? g[at] : 1.f;
      bn0 = t0 < n ? beta[at] : 0.f;
      gn1 = t0 + 1 < n ? g[at + Hv] : 1.f;
      bn1 = t0 + 1 < n ? beta[at + Hv] : 0.f;
    };
    auto make_gates = [&](float* gs) {  // one inclusive scan over token pairs
      const float lg0 = log2f(fminf(fmaxf(gn0, 1e-6f), 1.f));
      const float lg1 = log2f(fminf(fmaxf(gn1, 1e-6f), 1.f));
      const float pair = lg0 + lg1;
      float incl = pair;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane_id >= off) incl += y;
      }
      const float p0 = (incl - pair) + lg0, p1 = p0 + lg1;
      const float last = __shfl_sync(0xffffffffu, incl, 31);
      const float first = __shfl_sync(0xffffffffu, p0, 0);
      const int t0 = 2 * lane_id;
      gs[t0] = p0;
      gs[t0 + 1] = p1;
      gs[64 + t0] = bn0;
      gs[64 + t0 + 1] = bn1;
      gs[128 + t0] = exp2f(p0);
      gs[128 + t0 + 1] = exp2f(p1);
      gs[192 + t0] = exp2f(last - p0);
      gs[192 + t0 + 1] = exp2f(last - p1);
      gs[256 + t0] = exp2f(first - p0);
      gs[256 + t0 + 1] = exp2f(first - p1);
    };
    // A rows (lanes 0-63) in fp32 smem and m rows (lanes 64-127) as bf16 hi/lo
    // pair columns in TMEM cols T_M, from KK^T / QK^T (cols T_KK) and gate set gs;
    // columns [32 hx, 32 hx + 32) of this warp's lane quarter.
    auto build_am = [&](const float* gs, int hx) {
      float v[32];
      tc::tmem_ld32(tmem + lane + T_KK + 32 * hx, v);
      const int t = row & 63;
      const float lgt = gs[t];
      // R_tj = 2^(lg_t - lg_j). When the chunk's decay spans < 2^-100, write it
      // as 2^(lg_t - lg_0) * 2^(lg_0 - lg_j): both factors stay in range and the
      // per-element exponentials become one multiply.
      float rr[32];
      if (gs[0] - gs[63] < 100.f) {  // uniform over the CTA
        const float at = exp2f(lgt - gs[0]);
#pragma unroll
        for (int e = 0; e < 32; ++e) rr[e] = at * gs[256 + 32 * hx + e];
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) rr[e] = exp2f(lgt - gs[32 * hx + e]);
      }
      if (quarter < 2) {
        const float bt = gs[64 + t];
        float4* arow = reinterpret_cast<float4*>(Xf + t * kAStride + 32 * hx);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          float a[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 32 * hx + 4 * j4 + e;
            a[e] = j < t ? bt * rr[4 * j4 + e] * v[4 * j4 + e] : 0.f;
          }
          arow[j4] = make_float4(a[0], a[1], a[2], a[3]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = 32 * hx + e;
          v[e] = j <= t ? rr[e] * v[e] : 0.f;
        }
        tmem_store_hilo(tmem + lane + T_M + 16 * hx, tmem + lane + T_M + 32 + 16 * hx, v);
      }
    };
    int kq_ok = 1;
    // G0 of a chunk: [K;Q] K^T -> TMEM cols T_KK (lanes 0-63 KK^T, 64-127 QK^T), by
    // the prep's first thread once the chunk's K/Q tiles have landed. The commit
    // arrives even without the G0, so no thread waits in vain.
    auto issue_g0 = [&](int chunk) {
      const int bi = chunk % kKQBufs;
      kq_ok = mbar_wait_bounded(&bar_kq[bi], (chunk / kKQBufs) & 1, status) ? 1 : 0;
      if (kq_ok) {
        tc::fence_after();
        const uint32_t kq = OFF_KQ + bi * KQ_BYTES;
        constexpr uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t a = smem_addr(sm + kq + kb * 16384) + ks * 32;
            tc::mma_bf16(tmem + T_KK, tc::desc_kmajor(a), tc::desc_kmajor(a), id,
                         (kb | ks) != 0);
          }
      }
      tc::commit(bar_g0);
    };
    if (warp == 8) {
      fetch_gates(0);
      make_gates(gate_sets);
      if (1 < nchunks) fetch_gates(1);
    }
    if (ptid == 0) issue_g0(0);
    g0_pending = 1;
#pragma unroll 1
    for (int n = 0; n < nchunks; ++n) {
      // m (cols T_M) and the fp32 A / X scratch are free once the state chain's X
      // split and Y of chunk n - 1 have read them.
      if (n >= 1) {
        const int done = mbar_wait_bounded(bar_mfree, (n - 1) & 1, status) ? 1 : 0;
        ok = group_sync_and(kPrepBar, kPrepThreads, done && ok);
        if (!ok) break;
        tc::fence_after();
      }
      const float* gs = gate_sets + (n % kGateSets) * kGateSet;
      // This chunk's G0 went out after the previous chunk's A / m (or before the
      // loop), and its gate set at the end of the previous iteration.
      {
        const int done = mbar_wait_bounded(bar_g0, g0_phase, status) ? 1 : 0;
        if (done) {
          g0_phase ^= 1;
          g0_pending = 0;
        }
        ok = group_sync_and(kPrepBar, kPrepThreads, done && ok && kq_ok);
        if (!ok) break;
        tc::fence_after();
      }
#pragma unroll 1
      for (int hx = 0; hx < 2; ++hx) build_am(gs, hx);
      tc::tmem_wait_st();
      tc::fence_before();
      group_sync(kPrepBar, kPrepThreads);
      // The next chunk's G0, now that every prep warp has read T_KK.
      if (n + 1 < nchunks) {
        if (ptid == 0) {
          tc::fence_after();
          issue_g0(n + 1);
        }
        g0_pending = 1;
      }

      // X = (I + A)^-1 in place: 8 x 8 diagonal blocks by substitution, then the
      // off-diagonal blocks level by level (8, 16, 32 wide).
      // L0: warp pw inverts diagonal blocks pw (lanes 0-7) and pw + 4 (lanes 8-15);
      //     lane c8 of a block owns column c8.
      {
        const int c8 = lane_id & 7;
        const int blk = pw + 4 * ((lane_id >> 3) & 1);
        const float* Ab = Xf + (8 * blk) * kAStride + 8 * blk;
        // Right-looking substitution: once x[k] is final it updates every later
        // row, so the loads of column k do not wait on the x chain.
        float x[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) x[r] = (r == c8) ? 1.f : 0.f;
#pragma unroll
        for (int k = 0; k < 7; ++k) {
          float col[8];
#pragma unroll
          for (int r = k + 1; r < 8; ++r) col[r] = Ab[r * kAStride + k];
#pragma unroll
          for (int r = k + 1; r < 8; ++r) x[r] = fmaf(-col[r], x[k], x[r]);
        }
        __syncwarp();
        if (lane_id < 16) {
          float* Xb = Xf + (8 * blk) * kAStride + 8 * blk + c8;
#pragma unroll
          for (int r = 0; r < 8; ++r) Xb[r * kAStride] = x[r];
        }
      }
      group_sync(kPrepBar, kPrepThreads);
      // L0b: in each 16 x 16 diagonal block b, X[lower 8][upper 8] =
      //      -D_hi (A[lower 8][upper 8] D_lo); two outputs per thread.
      {
        float tsum[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int idx = ptid + kPrepThreads * i;
          const int bb = idx >> 6, r = (idx >> 3) & 7, cc = idx & 7;
          const int lo = 16 * bb, hi = 16 * bb + 8;
          const float* Arow = Xf + (hi + r) * kAStride + lo;
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) acc = fmaf(Arow[k], Xf[(lo + k) * kAStride + lo + cc], acc);
          tsum[i] = acc;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) Tbuf[ptid + kPrepThreads * i] = tsum[i];
        group_sync(kPrepBar, kPrepThreads);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int idx = ptid + kPrepThreads * i;
          const int bb = idx >> 6, r = (idx >> 3) & 7, cc = idx & 7;
          const int lo = 16 * bb, hi = 16 * bb + 8;
          const float* Drow = Xf + (hi + r) * kAStride + hi;
          float xs = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) xs = fmaf(Drow[k], Tbuf[bb * 64 + k * 8 + cc], xs);
          Xf[(hi + r) * kAStride + lo + cc] = -xs;
        }
      }
      group_sync(kPrepBar, kPrepThreads);
      // The off-diagonal blocks are products of the blocks already inverted, run
      // as warp tensor-core tiles (three tf32 products each, fp32-accurate): a
      // 16 x 8 output tile per warp and step, the intermediate in Tbuf (row
      // stride kTStride).
      // L1: X[2p+1][2p] = -D_{2p+1} (A[2p+1][2p] D_{2p}), p = 0, 1; warp pw owns
      //     p = pw / 2 and columns 8 (pw % 2) + [0, 8).
      {
        const int gq = lane_id >> 2, t4 = lane_id & 3;
        const int p = pw >> 1, n0 = 8 * (pw & 1);
        const int r1 = 16 * (2 * p + 1), c1 = 16 * (2 * p);
        float* T = Tbuf + p * 16 * kTStride + n0;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        warp_gemm_tf32x3<16>(acc, Xf + r1 * kAStride + c1, kAStride,
                             Xf + c1 * kAStride + c1 + n0, kAStride, lane_id);
        *reinterpret_cast<float2*>(T + gq * kTStride + 2 * t4) = make_float2(acc[0], acc[1]);
        *reinterpret_cast<float2*>(T + (gq + 8) * kTStride + 2 * t4) =
            make_float2(acc[2], acc[3]);
        group_sync(kPrepBar, kPrepThreads);
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        warp_gemm_tf32x3<16>(acc, Xf + r1 * kAStride + r1, kAStride, T, kTStride, lane_id);
        float* Xo = Xf + r1 * kAStride + c1 + n0;
        *reinterpret_cast<float2*>(Xo + gq * kAStride + 2 * t4) = make_float2(-acc[0], -acc[1]);
        *reinterpret_cast<float2*>(Xo + (gq + 8) * kAStride + 2 * t4) =
            make_float2(-acc[2], -acc[3]);
      }
      group_sync(kPrepBar, kPrepThreads);
      // L2: X[32:64][0:32] = -X[32:64][32:64] (A[32:64][0:32] X[0:32][0:32]); warp pw
      //     owns columns 8 pw + [0, 8) of row blocks 32 + [0, 16) and 48 + [0, 16).
      {
        const int gq = lane_id >> 2, t4 = lane_id & 3;
        const int n0 = 8 * pw;
        float acc[2][4];
#pragma unroll 1
        for (int i = 0; i < 2; ++i) {
          const int r0 = 32 + 16 * i;
          float* T = Tbuf + (r0 - 32) * kTStride + n0;
          acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
          warp_gemm_tf32x3<32>(acc[i], Xf + r0 * kAStride, kAStride, Xf + n0, kAStride, lane_id);
          *reinterpret_cast<float2*>(T + gq * kTStride + 2 * t4) = make_float2(acc[i][0], acc[i][1]);
          *reinterpret_cast<float2*>(T + (gq + 8) * kTStride + 2 * t4) =
              make_float2(acc[i][2], acc[i][3]);
        }
        group_sync(kPrepBar, kPrepThreads);  // T complete; every warp is done reading A[32:64][0:32]
#pragma unroll 1
        for (int i = 0; i < 2; ++i) {
          const int r0 = 32 + 16 * i;
          acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
          warp_gemm_tf32x3<32>(acc[i], Xf + r0 * kAStride + 32, kAStride, Tbuf + n0, kTStride,
                               lane_id);
          float* Xo = Xf + r0 * kAStride + n0;
          *reinterpret_cast<float2*>(Xo + gq * kAStride + 2 * t4) =
              make_float2(-acc[i][0], -acc[i][1]);
          *reinterpret_cast<float2*>(Xo + (gq + 8) * kAStride + 2 * t4) =
              make_float2(-acc[i][2], -acc[i][3]);
        }
      }
      group_sync(kPrepBar, kPrepThreads);
      if (ptid == 0) mbar_arrive(&bar_full[n & 1]);
      // The next chunk's gate set goes where chunk n - 2's was; the state chain
      // finished that chunk before its Y of chunk n - 1.
      if (warp == 8 && n + 1 < nchunks) {
        make_gates(gate_sets + ((n + 1) % kGateSets) * kGateSet);
        if (n + 2 < nchunks) fetch_gates(n + 2);
      }
    }
    // A bounded wait gave up: let this group's G0 in flight finish.
    if (g0_pending) mbar_wait_bounded(bar_g0, g0_phase, status);
  } else {
    // ================= the state chain of chunk c (warps 0-7).
    // Initial state: row i, columns [64 hf, 64 hf + 64) -> TMEM.
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      float v[32];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 x = reinterpret_cast<const float4*>(srow + 32 * q)[e];
        v[4 * e] = x.x;
        v[4 * e + 1] = x.y;
        v[4 * e + 2] = x.z;
        v[4 * e + 3] = x.w;
      }
      tc::tmem_st32(tmem + lane + T_S + 64 * hf + 32 * q, v);
    }
    tc::tmem_wait_st();

    uint32_t mma_phase = 0;
    int pending_mma = 0;
    // Loads in flight, for the drain on the error path: bit b = K/Q buffer b,
    // bit 3 = V; kq_last[b] / v_last = the chunk last loaded there.
    int pending_loads = 0;
    int kq_last[kKQBufs];
#pragma unroll
    for (int i = 0; i < kKQBufs; ++i) kq_last[i] = -1;
    int v_last = -1;
    if (tid == 0) {
      for (int i = 0; i < kKQBufs && i < nchunks; ++i) issue_kq(i);
      issue_v(0);
    }
    for (int i = 0; i < kKQBufs && i < nchunks; ++i) {
      pending_loads |= 1 << i;
      kq_last[i] = i;
    }
    pending_loads |= 8;
    v_last = 0;
    auto wait_mma = [&]() {
      const int done = mbar_wait_bounded(bar_mma, mma_phase, status) ? 1 : 0;
      if (done) {
        mma_phase ^= 1;
        pending_mma = 0;
      }
      ok = group_sync_and(kMainBar, kMainThreads, done && ok);
      tc::fence_after();
      return ok;
    };

#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
      const int tok0 = start + c * kC;
      const int valid = min(kC, len - c * kC);
      const int bi = c % kKQBufs;
      const uint32_t off_kq = OFF_KQ + bi * KQ_BYTES;
      uint8_t* xyh = sm + OFF_XYH;
      uint8_t* xyl = sm + OFF_XYL;
      const float* s_lg = gate_sets + (c % kGateSets) * kGateSet;
      const float* s_beta = s_lg + 64;
      const float* s_decay = s_lg + 128;
      const float* s_r = s_lg + 192;

      // ---- (1) this chunk's prep: gate set, m in cols T_M, X in the fp32 scratch;
      //          and (thread 0) its K/Q tiles, which the prep's G0 waited for.
      {
        int done = mbar_wait_bounded(&bar_full[c & 1], (c >> 1) & 1, status) ? 1 : 0;
        if (tid == 0 && done) done = mbar_wait_bounded(&bar_kq[bi], (c / kKQBufs) & 1, status);
        ok = group_sync_and(kMainBar, kMainThreads, done && ok);
        if (!ok) break;
        tc::fence_after();
        pending_loads &= ~(1 << bi);
      }
      // ---- (4b) X -> bf16 hi/lo: X^T rows (B of Y) and X rows (rows 0-63 of
      //           [X;Y], B of G34; the previous chunk's G34 is done). Then the prep
      //           may overwrite the fp32 X (its other condition is Y's commit).
      {
        const int xj = tid & 63, xpart = tid >> 6;
        float xc[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) xc[e] = Xf[(16 * xpart + e) * kAStride + xj];
        store_chunk8_hilo(sm + OFF_XTH, sm + OFF_XTL, xj, 2 * xpart, xc);
        store_chunk8_hilo(sm + OFF_XTH, sm + OFF_XTL, xj, 2 * xpart + 1, xc + 8);
        const float4* xr = reinterpret_cast<const float4*>(Xf + xj * kAStride + 16 * xpart);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 x4 = xr[e];
          xc[4 * e] = x4.x;
          xc[4 * e + 1] = x4.y;
          xc[4 * e + 2] = x4.z;
          xc[4 * e + 3] = x4.w;
        }
        store_chunk8_hilo(xyh, xyl, xj, 2 * xpart, xc);
        store_chunk8_hilo(xyh, xyl, xj, 2 * xpart + 1, xc + 8);
      }
      fence_proxy_async_smem();
      group_sync(kMainBar, kMainThreads);
      if (tid == 0) mbar_arrive(bar_mfree);

      // ---- (5) Y = m X, m from TMEM cols T_M (lanes 64-127: hi, then lo) -> TMEM
      //          cols T_P (lanes 64-127; G12 writes them next). Lanes 0-63 of the
      //          product are not used. A second commit tells the prep that m has
      //          been read.
      if (tid == 0) {
        tc::fence_after();
        constexpr uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t mh = tmem + T_M + 8 * ks, ml = tmem + T_M + 32 + 8 * ks;
          const uint64_t xh = tc::desc_kmajor(smem_addr(sm + OFF_XTH) + ks * 32);
          const uint64_t xl = tc::desc_kmajor(smem_addr(sm + OFF_XTL) + ks * 32);
          tc::mma_bf16_ts(tmem + T_P, mh, xh, id, ks != 0);
          tc::mma_bf16_ts(tmem + T_P, mh, xl, id, true);
          tc::mma_bf16_ts(tmem + T_P, ml, xh, id, true);
        }
        tc::commit(bar_mma);
        tc::commit(bar_mfree);
      }
      pending_mma = 1;
      // ---- (6) S hi/lo (A of G12) -> TMEM cols T_SH / T_SL while Y runs (Y reads
      //          the T_M and writes the T_P columns; S was last written by the
      //          previous chunk's GS, which has finished reading T_SH / T_SL).
      //          Columns [64 hf, +64) of S -> bf16 pair columns [32 hf, +32).
#pragma unroll 1
      for (int q = 0; q < 2; ++q) {
        float v[32];
        tc::tmem_ld32(tmem + lane + T_S + 64 * hf + 32 * q, v);
        tmem_store_hilo(tmem + lane + T_SH + 32 * hf + 16 * q,
                        tmem + lane + T_SL + 32 * hf + 16 * q, v);
      }
      tc::tmem_wait_st();
      if (!wait_mma()) break;
      if (quarter >= 2) {
        float y[32];
        tc::tmem_ld32(tmem + lane + T_P + 32 * hf, y);
        store_chunks_hilo(xyh, xyl, row, 4 * hf, y);
      }
      fence_proxy_async_smem();
      tc::fence_before();
      group_sync(kMainBar, kMainThreads);

      // ---- (7) G12: S [K;Q]^T -> TMEM cols T_P.
      if (tid == 0) {
        tc::fence_after();
        constexpr uint32_t id = tc::idesc_bf16(128, 128, false, false);
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint32_t a = tmem + (part ? T_SL : T_SH) + 32 * kb + 8 * ks;
              const uint32_t bb = smem_addr(sm + off_kq + kb * 16384) + ks * 32;
              tc::mma_bf16_ts(tmem + T_P, a, tc::desc_kmajor(bb), id, (part | kb | ks) != 0);
            }
        tc::commit(bar_mma);
      }
      pending_mma = 1;
      // ---- (6b) decay_63 * S -> TMEM while G12 runs (G12 reads the T_SH / T_SL
      //           columns and writes the T_P columns only).
      {
        const float dl = s_decay[63];
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          float v[32];
          const uint32_t col = T_S + 64 * hf + 32 * q;
          tc::tmem_ld32(tmem + lane + col, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= dl;
          tc::tmem_st32(tmem + lane + col, v);
        }
        tc::tmem_wait_st();
        tc::fence_before();
      }
      if (!wait_mma()) break;

      // ---- (8) W^T row i for tokens [32 hf, +32) -> TMEM cols T_SH / T_SL as
      //          bf16 hi/lo (the A operand of G34; G12 has finished reading S
      //          there); zero those U^T columns; decay * P2^T in the matching O^T
      //          columns.
      {
        const int done = mbar_wait_bounded(bar_v, c & 1, status) ? 1 : 0;
        ok = group_sync_and(kMainBar, kMainThreads, done && ok);
        if (!ok) break;
        pending_loads &= ~8;
      }
      {
        float p[32];
        tc::tmem_ld32(tmem + lane + T_P + 32 * hf, p);
        const uint8_t* vt = sm + OFF_V + (row >> 6) * 8192;
        const int iv = row & 63;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int t = 32 * hf + e;
          const float vti = bf16_to_f(*reinterpret_cast<const uint16_t*>(vt + tc::swz(t, iv)));
          p[e] = s_beta[t] * (vti - s_decay[t] * p[e]);
        }
        tmem_store_hilo(tmem + lane + T_SH + 16 * hf, tmem + lane + T_SL + 16 * hf, p);
        float z[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) z[e] = 0.f;
        tc::tmem_st32(tmem + lane + T_P + 32 * hf, z);
        tc::tmem_ld32(tmem + lane + T_P + 64 + 32 * hf, p);
#pragma unroll
        for (int e = 0; e < 32; ++e) p[e] *= s_decay[32 * hf + e];
        tc::tmem_st32(tmem + lane + T_P + 64 + 32 * hf, p);
        tc::tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc::fence_before();
      group_sync(kMainBar, kMainThreads);
      if (c + 1 < nchunks) {  // every thread has read this chunk's V; warp 3 loads the next
        if (tid == 96) issue_v(c + 1);
        pending_loads |= 8;
        v_last = c + 1;
      }

      // ---- (9) G34: W^T [X;Y]^T accumulated -> U^T | O^T.
      if (tid == 0) {
        tc::fence_after();
        constexpr uint32_t id = tc::idesc_bf16(128, 128, false, false);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t wh = tmem + T_SH + 8 * ks, wl = tmem + T_SL + 8 * ks;
          const uint64_t xh = tc::desc_kmajor(smem_addr(xyh) + ks * 32);
          const uint64_t xl = tc::desc_kmajor(smem_addr(xyl) + ks * 32);
          tc::mma_bf16_ts(tmem + T_P, wh, xh, id, true);
          tc::mma_bf16_ts(tmem + T_P, wh, xl, id, true);
          tc::mma_bf16_ts(tmem + T_P, wl, xh, id, true);
        }
        tc::commit(bar_mma);
      }
      pending_mma = 1;
      if (!wait_mma()) break;

      // ---- (10) (U^T r) hi/lo -> TMEM cols T_SH / T_SL (the A operand of GS; G34
      //           has finished reading W there) for tokens [32 hf, +32).
      {
        float u[32];
        tc::tmem_ld32(tmem + lane + T_P + 32 * hf, u);
#pragma unroll
        for (int e = 0; e < 32; ++e) u[e] *= s_r[32 * hf + e];
        tmem_store_hilo(tmem + lane + T_SH + 16 * hf, tmem + lane + T_SL + 16 * hf, u);
        tc::tmem_wait_st();
      }
      tc::fence_before();
      group_sync(kMainBar, kMainThreads);

      // ---- (11) GS: S += (U^T r) K, K as an MN-major operand (dk halves 16 KiB apart).
      if (tid == 0) {
        tc::fence_after();
        constexpr uint32_t id = tc::idesc_bf16(128, 128, false, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t kd = tc::desc_mnmajor(smem_addr(sm + off_kq) + ks * 2048, 16384);
          tc::mma_bf16_ts(tmem + T_S, tmem + T_SH + 8 * ks, kd, id, true);
          tc::mma_bf16_ts(tmem + T_S, tmem + T_SL + 8 * ks, kd, id, true);
        }
        tc::commit(bar_mma);
      }
      pending_mma = 1;
      // ---- (10b) O^T -> out (bf16) for tokens [32 hf, +32) while GS runs (it
      //            writes the T_S columns only).
      {
        float o[32];
        tc::tmem_ld32(tmem + lane + T_P + 64 + 32 * hf, o);
        uint16_t* orow = out + ((size_t)(tok0 + 32 * hf) * Hv + h) * kD + row;
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (32 * hf + e < valid) orow[(size_t)e * Hv * kD] = f_to_bf16(o[e]);
      }
      if (!wait_mma()) break;
      // This chunk's K/Q buffer is free (its G0, G12 and GS are done): warp 3
      // fetches chunk c + kKQBufs into it.
      if (c + kKQBufs < nchunks) {
        if (tid == 96) issue_kq(c + kKQBufs);
        pending_loads |= 1 << bi;
        kq_last[bi] = c + kKQBufs;
      }
    }

    if (!ok) {
      // A bounded wait gave up (already flagged): let this CTA's own copies and
      // MMAs in flight finish, within limits, before the TMEM is released.
      if (tid == 0) {
        for (int b2 = 0; b2 < kKQBufs; ++b2)
          if ((pending_loads & (1 << b2)) && kq_last[b2] >= 0)
            mbar_wait_bounded(&bar_kq[b2], (kq_last[b2] / kKQBufs) & 1, status);
        if ((pending_loads & 8) && v_last >= 0) mbar_wait_bounded(bar_v, v_last & 1, status);
      }
      if (pending_mma) mbar_wait_bounded(bar_mma, mma_phase, status);
    } else {
#pragma unroll 1
      for (int q = 0; q < 2; ++q) {
        float v[32];
        tc::tmem_ld32(tmem + lane + T_S + 64 * hf + 32 * q, v);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          reinterpret_cast<float4*>(srow + 32 * q)[e] =
              make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [tokens][heads][128] bf16 viewed as a 3-D tensor (d, head, token); box 64 x 1 x 64.
int encode_rows(CUtensorMap* map, const void* base, int heads, long long tokens,
                const char* what) {
  auto fn = encode_fn();
  if (fn == nullptr)
    return set_error(SC_ERR_CUDA, "sc_gdn_chunk_prefill: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)heads * kD * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kC};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                  strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SC_ERR_INVALID, "sc_gdn_chunk_prefill: tensor map for %s rejected (%d)",
                     what, (int)r);
  return SC_OK;
}

}  // namespace
}  // namespace sc

extern "C" int sc_gdn_chunk_prefill(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                                    const float* g, const float* beta, float* state,
                                    const int32_t* state_slot, const int32_t* cu_seqlens,
                                    sc_bf16* out, int B, int T, int total_tokens, int Hk, int Hv,
                                    int dk, int dv, int num_slots, void* stream) {
  const char* name = "sc_gdn_chunk_prefill";
  SC_REQUIRE(q && k && v && g && beta && state && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(dk == sc::kD && dv == sc::kD, SC_ERR_UNSUPPORTED, "%s: dk=%d dv=%d (only 128x128)",
             name, dk, dv);
  SC_REQUIRE(B >= 0 && Hk > 0 && Hv > 0 && Hv % Hk == 0, SC_ERR_INVALID,
             "%s: bad heads B=%d Hk=%d Hv=%d", name, B, Hk, Hv);
  SC_REQUIRE((long long)B * Hv < (1LL << 31), SC_ERR_INVALID, "%s: B*Hv too large", name);
  SC_REQUIRE(num_slots > 0 && (state_slot != nullptr || num_slots >= B), SC_ERR_INVALID,
             "%s: num_slots=%d for B=%d", name, num_slots, B);
  long long tokens;
  if (cu_seqlens == nullptr) {
    SC_REQUIRE(T >= 0, SC_ERR_INVALID, "%s: T=%d", name, T);
    tokens = (long long)B * T;
  } else {
    SC_REQUIRE(total_tokens >= 0, SC_ERR_INVALID, "%s: total_tokens=%d", name, total_tokens);
    tokens = total_tokens;
  }
  if (B == 0 || tokens == 0) return SC_OK;
  SC_REQUIRE(tokens < (1LL << 31), SC_ERR_INVALID, "%s: too many tokens", name);
  SC_REQUIRE(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0, SC_ERR_INVALID,
             "%s: q/k/v must be 16-byte aligned", name);
  CUtensorMap tq, tk, tv;
  if (int rc = sc::encode_rows(&tq, q, Hk, tokens, "q")) return rc;
  if (int rc = sc::encode_rows(&tk, k, Hk, tokens, "k")) return rc;
  if (int rc = sc::encode_rows(&tv, v, Hv, tokens, "v")) return rc;

  static int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(sc::gdn_chunk_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)sc::SMEM_BYTES);
    if (err != cudaSuccess)
      return sc::set_error(SC_ERR_CUDA, "%s: smem attribute: %s", name, cudaGetErrorString(err));
    configured[dev] = 1;
  }
  sc::gdn_chunk_kernel<<<B * Hv, sc::kThreads, sc::SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
      tq, tk, tv, g, beta, state, state_slot, cu_seqlens, out, Hk, Hv, T, num_slots,
      sc::device_status_word());
  return sc::check_launch(name);
}
