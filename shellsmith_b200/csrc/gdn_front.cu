// GDN layer glue fused around the recurrence: causal-conv taps, SiLU, q/k
// normalisation, gates, and the gated RMS norm of the output.
//
// Reference: studio_compute/numerics/bf16.py:44-139 (`gdn_inner`, the branch
// decode_one=True takes) and :191-210 (`_decode_gdn_token`). Per layer and row:
//   conv   = silu(depthwise_conv_K4([taps; qkv]))         bf16.py:78-79
//   q,k,v  = split(conv);  q = rms_norm(q)/dk, k = rms_norm(k)/sqrt(dk)
//   beta   = sigmoid(b);  g = exp(-exp(A_log) * softplus(a + dt_bias))   :98-102
//   y      = gated_delta_token(q, k, v, g, beta, S)        :103-108
//   out    = rms_norm(y, w, eps) * silu(z)                 :129-135
//   taps   = last 3 rows of [taps; qkv]                    :137
// Every MLX op on bf16 arrays rounds its result to bf16; these kernels compute
// in fp32 and round at the same points, so their values are the ones the
// reference's unfused decode path hands from op to op.
//
// Tap storage. The reference carries taps[B, 3, C] and rebuilds it each step.
// Here each state slot owns a ring of 4 rows, taps[slot][4][C]: the token at
// absolute position t reads rows (t-3)&3, (t-2)&3, (t-1)&3 and writes its own
// input into row t&3, which no reader of step t touches. So many CTAs can
// share one key head's channels with no ordering between them and one row
// (2*C bytes) is written per token instead of three.
//
// K8 gdn_decode_fused: the bulk-copy state update of gdn_decode.cu with the
// front computed while the state chunks are in flight, and the gated RMS norm
// as its epilogue. The norm spans all 128 value rows of a head, which two CTAs
// (64 rows each) share: they form a 2-CTA cluster and exchange their partial
// sums of squares through distributed shared memory.
// K9 gdn_prefill_front: the same front for the packed tokens of a prefill, to
// feed sc_gdn_chunk_prefill; K10 gdn_taps_store writes each prompt's last
// three inputs into its ring afterwards; K11 gated_rmsnorm is the output norm
// for any number of rows.
#include <algorithm>

#include "common.cuh"
#include "gdn_internal.cuh"

namespace sc {
namespace {

constexpr int kHead = 128;                       // dk = dv = 128
constexpr int kRing = 4;                         // tap ring rows per slot
constexpr int kFRows = 32;                       // state rows per bulk chunk
constexpr int kFChunkBytes = kFRows * kHead * 4;  // 16 KiB
constexpr int kFChunks = 2;                      // 64 value rows per CTA
constexpr int kTokTile = 16;                     // prefill tokens per CTA
constexpr int kTokTileDecode = 4;                // one-token rows per CTA (decode batches)

__device__ __forceinline__ float bfr(float x) { return bf16_to_f(f_to_bf16(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float silu_bf(float x) { return bfr(x * bfr(sigmoid_f(x))); }
__device__ __forceinline__ float softplus_f(float x) {
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// silu(conv) of channel c: history h0..h2 (oldest first), input x, weight row w[c][0..3].
__device__ __forceinline__ float conv_silu(const uint16_t* __restrict__ w, int c, float h0,
                                           float h1, float h2, float x) {
  const uint2 wv = __ldg(reinterpret_cast<const uint2*>(w + (size_t)c * 4));
  float y = bf16_lo(wv.x) * h0;
  y = fmaf(bf16_hi(wv.x), h1, y);
  y = fmaf(bf16_lo(wv.y), h2, y);
  y = fmaf(bf16_hi(wv.y), x, y);
  return silu_bf(bfr(y));
}

// g and beta of one (token, head) from the logits, each op rounded like the reference.
__device__ __forceinline__ void make_gates(float a, float b, float a_log, float dt_bias,
                                           float& g, float& beta) {
  const float x = bfr(bfr(a) + bfr(dt_bias));
  const float sp = bfr(softplus_f(x));
  const float rate = bfr(expf(bfr(a_log)));
  g = bfr(expf(bfr(-rate * sp)));
  beta = bfr(sigmoid_f(bfr(b)));
}

// Gates of the fused chunk path from their logits: the reference's sampler_gate
// and sampler_beta (numerics/metal/gdn_chunk_common.metal:61-75), which the
// chunk kernel behind gdn_fused.py:86-122 `gated_delta_chunks` makes per row.
// fp32 math rounded to bf16 after each step; softplus as max(x, 0) +
// log(1 + exp(-|x|)). The gate is returned as its bf16 value (not clamped: the
// chunk kernel clamps it at 1e-6 before its log, as the reference does).
__device__ __forceinline__ void sampler_gates(float a, float b, float a_log, float dt_bias,
                                              float& g, float& beta) {
  const float scale = bfr(expf(bfr(a_log)));
  const float x = bfr(a + bfr(dt_bias));
  const float sp = bfr(fmaxf(x, 0.f) + logf(1.f + expf(-fabsf(x))));
  g = bfr(expf(bfr(-scale * sp)));
  beta = bfr(1.f / (1.f + expf(-b)));
}

// One thread per (token, value head); a and b are [rows][Hv] bf16.
__global__ void __launch_bounds__(256)
    sampler_gates_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                         const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                         float* __restrict__ g, float* __restrict__ beta, long long n, int Hv) {
  pdl_wait();
  pdl_trigger();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int h = (int)(i % Hv);
    float gi, bi;
    sampler_gates(bf16_to_f(a[i]), bf16_to_f(b[i]), a_log[h], dt_bias[h], gi, bi);
    g[i] = gi;
    beta[i] = bi;
  }
}

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// A float in the shared memory of CTA `rank` of this cluster, at the address
// `p` has in this CTA.
__device__ __forceinline__ float ld_peer_f32(const float* p, uint32_t rank) {
  uint32_t local = smem_addr(p), remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

struct FusedSmem {
  float q[kHead], k[kHead], v[kFChunks * kFRows], o[kFChunks * kFRows];
  float red[8];
  float part;      // this CTA's sum of squares of its 64 outputs (read by the peer)
  float gate[2];   // g, beta
  unsigned int aborted;
  uint64_t bars[kFChunks];
};

__global__ void __cluster_dims__(1, 2, 1) __launch_bounds__(128)
    gdn_decode_fused_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ z,
                            const uint16_t* __restrict__ a_in, const uint16_t* __restrict__ b_in,
                            const uint16_t* __restrict__ conv_w, const float* __restrict__ a_log,
                            const float* __restrict__ dt_bias,
                            const uint16_t* __restrict__ norm_w, float eps,
                            uint16_t* __restrict__ taps, const int32_t* __restrict__ position,
                            float* __restrict__ state, const int32_t* __restrict__ state_slot,
                            uint16_t* __restrict__ out, int Hk, int Hv, int num_slots,
                            unsigned int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  FusedSmem& sm = *reinterpret_cast<FusedSmem*>(smem + kFChunks * kFChunkBytes);
  const int bh = blockIdx.x, half = blockIdx.y;
  const int b = bh / Hv, h = bh - b * Hv;
  const int slot = state_slot != nullptr ? state_slot[b] : b;
  const int t = position[b];
  // Both CTAs of a cluster share b, so these exits are taken by both or neither.
  if (slot < 0) return;
  if (slot >= num_slots || t < 0) {
    if (threadIdx.x == 0 && half == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ratio = Hv / Hk, kh = h / ratio;
  const size_t C = (size_t)(2 * Hk + Hv) * kHead;
  float* S = state + ((size_t)slot * Hv + h) * (size_t)kHead * kHead +
             (size_t)half * kFChunks * kFRows * kHead;
  if (tid == 0) {
    // One thread decides whether an earlier wait timed out, so the whole CTA
    // either streams its chunks or skips them (the cluster barriers still run).
    sm.aborted = status != nullptr &&
                 (*reinterpret_cast<volatile unsigned int*>(status) & DEV_WAIT_TIMEOUT);
    for (int c = 0; c < kFChunks; ++c) mbar_init(&sm.bars[c], 1);
    fence_mbar_init();
    if (!sm.aborted) {
      for (int c = 0; c < kFChunks; ++c) {
        mbar_arrive_expect_tx(&sm.bars[c], kFChunkBytes);
        bulk_g2s(smem + c * kFChunkBytes, S + (size_t)c * kFRows * kHead, kFChunkBytes,
                 &sm.bars[c]);
      }
    }
  }

  // ---- front, while the state chunks land. Every global load of the CTA is
  // issued here, so under a saturated memory system it pays one round trip.
  constexpr int kRowsCta = kFChunks * kFRows;
  const int row_out = half * kRowsCta + (tid & (kRowsCta - 1));
  const float z_row = bf16_to_f(z[(size_t)bh * kHead + row_out]);
  const float w_row = bf16_to_f(norm_w[row_out]);
  float ga = 0.f, gb = 0.f, galog = 0.f, gdt = 0.f;
  if (tid == 0) {
    ga = bf16_to_f(a_in[bh]);
    gb = bf16_to_f(b_in[bh]);
    galog = a_log[h];
    gdt = dt_bias[h];
  }
  const uint16_t* xrow = qkv + (size_t)b * C;
  uint16_t* ring = taps + (size_t)slot * kRing * C;
  const size_t r0 = (size_t)((t - 3) & 3) * C, r1 = (size_t)((t - 2) & 3) * C,
               r2 = (size_t)((t - 1) & 3) * C, rw = (size_t)(t & 3) * C;
  const bool tap_writer = (h % ratio == 0) && half == 0;
  float qv, kv;
  {
    const int cq = kh * kHead + tid, ck = (Hk + kh) * kHead + tid;
    const uint16_t xq = xrow[cq], xk = xrow[ck];
    qv = conv_silu(conv_w, cq, bf16_to_f(ring[r0 + cq]), bf16_to_f(ring[r1 + cq]),
                   bf16_to_f(ring[r2 + cq]), bf16_to_f(xq));
    kv = conv_silu(conv_w, ck, bf16_to_f(ring[r0 + ck]), bf16_to_f(ring[r1 + ck]),
                   bf16_to_f(ring[r2 + ck]), bf16_to_f(xk));
    if (tap_writer) {
      ring[rw + cq] = xq;
      ring[rw + ck] = xk;
    }
  }
  if (tid < kFChunks * kFRows) {
    const int cv = (2 * Hk + h) * kHead + half * kFChunks * kFRows + tid;
    const uint16_t xv = xrow[cv];
    sm.v[tid] = conv_silu(conv_w, cv, bf16_to_f(ring[r0 + cv]), bf16_to_f(ring[r1 + cv]),
                          bf16_to_f(ring[r2 + cv]), bf16_to_f(xv));
    ring[rw + cv] = xv;
    sm.o[tid] = 0.f;
  }
  if (tid == 0) make_gates(ga, gb, galog, gdt, sm.gate[0], sm.gate[1]);
  {
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      sm.red[warp] = sq;
      sm.red[4 + warp] = sk;
    }
  }
  __syncthreads();  // also publishes the barrier initialisation
  {
    const float mq = (sm.red[0] + sm.red[1] + sm.red[2] + sm.red[3]) * (1.f / kHead);
    const float mk = (sm.red[4] + sm.red[5] + sm.red[6] + sm.red[7]) * (1.f / kHead);
    const float inv_dk = bfr(1.f / kHead), inv_sqrt_dk = bfr(0.08838834764831845f);
    sm.q[tid] = bfr(bfr(qv * (1.f / sqrtf(mq + 1e-6f))) * inv_dk);
    sm.k[tid] = bfr(bfr(kv * (1.f / sqrtf(mk + 1e-6f))) * inv_sqrt_dk);
  }
  __syncthreads();

  // ---- state update (as gdn_decode_bulk_kernel), outputs kept in shared memory
  const float4 kf = reinterpret_cast<const float4*>(sm.k)[lane];
  const float4 qf = reinterpret_cast<const float4*>(sm.q)[lane];
  const float decay = sm.gate[0], bt = sm.gate[1];
  const bool aborted = sm.aborted != 0;
  int ok = aborted ? 0 : 1;
  for (int c = 0; c < kFChunks; ++c) {
    if (ok && !mbar_wait_bounded(&sm.bars[c], 0, status)) ok = 0;
    if (ok) {
      float4* rows = reinterpret_cast<float4*>(smem + c * kFChunkBytes);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int lr = 8 * warp + r;
        float4 s4 = rows[lr * 32 + lane];
        s4.x *= decay;
        s4.y *= decay;
        s4.z *= decay;
        s4.w *= decay;
        const float pred = warp_sum(s4.x * kf.x + s4.y * kf.y + s4.z * kf.z + s4.w * kf.w);
        const float delta = bt * (sm.v[c * kFRows + lr] - pred);
        s4.x = fmaf(delta, kf.x, s4.x);
        s4.y = fmaf(delta, kf.y, s4.y);
        s4.z = fmaf(delta, kf.z, s4.z);
        s4.w = fmaf(delta, kf.w, s4.w);
        const float o = warp_sum(s4.x * qf.x + s4.y * qf.y + s4.z * qf.z + s4.w * qf.w);
        rows[lr * 32 + lane] = s4;
        if (lane == 0) sm.o[c * kFRows + lr] = bfr(o);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0 && ok) {
      bulk_s2g(S + (size_t)c * kFRows * kHead, smem + c * kFChunkBytes, kFChunkBytes);
      bulk_commit();
    }
  }

  // ---- gated RMS norm over the head's 128 outputs: 64 here, 64 in the peer CTA
  {
    const float y = tid < kFChunks * kFRows ? sm.o[tid] : 0.f;
    const float s = warp_sum(y * y);
    if (lane == 0) sm.red[warp] = s;
  }
  __syncthreads();
  if (tid == 0) sm.part = sm.red[0] + sm.red[1];
  cluster_arrive();  // publishes sm.part to the peer
  cluster_wait();
  const float total = sm.part + ld_peer_f32(&sm.part, cluster_rank() ^ 1u);
  cluster_arrive();  // this CTA is done reading the peer's shared memory
  if (tid < kRowsCta) {
    const float rstd = 1.f / sqrtf(total * (1.f / kHead) + eps);
    const float nrm = bfr(sm.o[tid] * rstd * w_row);
    out[(size_t)bh * kHead + row_out] = f_to_bf16(nrm * silu_bf(z_row));
  }
  if (tid == 0) {
    if (!ok && !aborted) {
      for (int c = 0; c < kFChunks; ++c) mbar_wait_bounded(&sm.bars[c], 0, status);
    }
    bulk_wait_read_all();
  }
  cluster_wait();  // the peer has read this CTA's sm.part; shared memory may go
}

// ---------------------------------------------------------------- prefill front
struct Seq {
  int index, pos;  // sequence of a token, and its position inside the sequence
};

__device__ __forceinline__ Seq find_seq(const int32_t* __restrict__ cu, int nseq, int token) {
  int lo = 0, hi = nseq;  // cu[lo] <= token < cu[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(cu + mid) <= token) lo = mid;
    else hi = mid;
  }
  return {lo, token - __ldg(cu + lo)};
}

// grid (token tiles, 2*Hk + Hv channel blocks of 128), 128 threads: thread =
// channel of the block, looping over TILE tokens. Without cu_seqlens (a decode
// batch: row i is a one-token sequence at position seq_start[i], each row its
// own slot) the kernel also stores each row's input into ring row
// position & 3 of its slot; the reads of that row are of rows position-3..-1.
template <int TILE>
__global__ void __launch_bounds__(128)
    gdn_prefill_front_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ a_in,
                             const uint16_t* __restrict__ b_in,
                             const uint16_t* __restrict__ conv_w,
                             const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                             uint16_t* __restrict__ taps, const int32_t* __restrict__ cu,
                             const int32_t* __restrict__ seq_slot,
                             const int32_t* __restrict__ seq_start, uint16_t* __restrict__ q_out,
                             uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out,
                             float* __restrict__ g_out, float* __restrict__ beta_out, int nseq,
                             int total, int Hk, int Hv, int num_slots, unsigned int* status) {
  __shared__ float red[4][TILE];
  // Launched as a dependent of the kernel before it: nothing is touched before
  // that kernel has completed. A state update launched as this kernel's own
  // dependent may start streaming its state now; it reads this kernel's
  // outputs only after they land.
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int blk = blockIdx.y;
  const int c = blk * kHead + tid;
  const size_t C = (size_t)(2 * Hk + Hv) * kHead;
  const int i0 = blockIdx.x * TILE;
  const int kind = blk < Hk ? 0 : (blk < 2 * Hk ? 1 : 2);  // q, k, v block
  float val[TILE];
  // Sequence of the tile's first token by binary search, then a forward walk;
  // without cu_seqlens token i is sequence i (a decode batch).
  int seq = 0, seq_end = 0;
  if (cu != nullptr && i0 < total) {
    seq = find_seq(cu, nseq, i0).index;
    seq_end = __ldg(cu + seq + 1);
  }
#pragma unroll
  for (int j = 0; j < TILE; ++j) {
    const int i = i0 + j;
    val[j] = 0.f;
    if (i >= total) continue;
    Seq sq;
    if (cu == nullptr) {
      sq = {i, 0};
    } else {
      while (i >= seq_end) seq_end = __ldg(cu + (++seq) + 1);
      sq = {seq, i - __ldg(cu + seq)};
    }
    const int slot = seq_slot != nullptr ? __ldg(seq_slot + sq.index) : sq.index;
    const int start = __ldg(seq_start + sq.index);
    if (slot < 0) continue;  // an inactive row (decode batches): no history, outputs unused
    if (slot >= num_slots || start < 0) {
      if (tid == 0) flag_device(status, DEV_BAD_INDEX);
      continue;
    }
    uint16_t* ring = taps + (size_t)slot * kRing * C;
    float hist[3];
#pragma unroll
    for (int d = 3; d >= 1; --d) {
      hist[3 - d] = sq.pos - d >= 0
                        ? bf16_to_f(qkv[(size_t)(i - d) * C + c])
                        : bf16_to_f(ring[(size_t)((start + sq.pos - d) & 3) * C + c]);
    }
    const uint16_t x = qkv[(size_t)i * C + c];
    val[j] = conv_silu(conv_w, c, hist[0], hist[1], hist[2], bf16_to_f(x));
    if (cu == nullptr) ring[(size_t)(start & 3) * C + c] = x;
  }
  if (kind == 2) {
    const int h = blk - 2 * Hk;
#pragma unroll
    for (int j = 0; j < TILE; ++j) {
      const int i = i0 + j;
      if (i < total) v_out[((size_t)i * Hv + h) * kHead + tid] = f_to_bf16(val[j]);
    }
    if (tid < TILE && i0 + tid < total) {
      const size_t e = (size_t)(i0 + tid) * Hv + h;
      float g, beta;
      make_gates(bf16_to_f(a_in[e]), bf16_to_f(b_in[e]), a_log[h], dt_bias[h], g, beta);
      g_out[e] = g;
      beta_out[e] = beta;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < TILE; ++j) {
    const float s = warp_sum(val[j] * val[j]);
    if (lane == 0) red[warp][j] = s;
  }
  __syncthreads();
  const int head = kind == 0 ? blk : blk - Hk;
  uint16_t* dst = kind == 0 ? q_out : k_out;
  const float scale = kind == 0 ? bfr(1.f / kHead) : bfr(0.08838834764831845f);
#pragma unroll
  for (int j = 0; j < TILE; ++j) {
    const int i = i0 + j;
    if (i >= total) continue;
    const float m = (red[0][j] + red[1][j] + red[2][j] + red[3][j]) * (1.f / kHead);
    dst[((size_t)i * Hk + head) * kHead + tid] =
        f_to_bf16(bfr(val[j] * (1.f / sqrtf(m + 1e-6f))) * scale);
  }
}

// The front for a decode batch (row i is one token at position seq_start[i]):
// one warp per (row, head) with four channels per lane, so every access is an
// 8-byte vector and the q/k L2 norm is one warp sum. The arithmetic and
// rounding points are those of gdn_prefill_front_kernel (only the order of the
// norm's sum differs). Reads ring rows (start-3..start-1) & 3 of the row's slot
// and stores the input into row start & 3.
__global__ void __launch_bounds__(128)
    gdn_decode_front_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ a_in,
                            const uint16_t* __restrict__ b_in,
                            const uint16_t* __restrict__ conv_w,
                            const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                            uint16_t* __restrict__ taps, const int32_t* __restrict__ seq_slot,
                            const int32_t* __restrict__ seq_start, uint16_t* __restrict__ q_out,
                            uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out,
                            float* __restrict__ g_out, float* __restrict__ beta_out, int B,
                            int Hk, int Hv, int num_slots, unsigned int* status) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int nh = 2 * Hk + Hv;
  const long long item = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (item >= (long long)B * nh) return;
  const int i = (int)(item / nh), blk = (int)(item - (long long)i * nh);
  const size_t C = (size_t)nh * kHead;
  const int c0 = blk * kHead + 4 * lane;
  const int slot = seq_slot != nullptr ? __ldg(seq_slot + i) : i;
  const int start = __ldg(seq_start + i);
  float val[4] = {0.f, 0.f, 0.f, 0.f};
  bool active = slot >= 0;  // an inactive row: no history, outputs unused
  if (active && (slot >= num_slots || start < 0)) {
    if (lane == 0) flag_device(status, DEV_BAD_INDEX);
    active = false;
  }
  if (active) {
    uint16_t* ring = taps + (size_t)slot * kRing * C + c0;
    const uint2 h0 = *reinterpret_cast<const uint2*>(ring + (size_t)((start - 3) & 3) * C);
    const uint2 h1 = *reinterpret_cast<const uint2*>(ring + (size_t)((start - 2) & 3) * C);
    const uint2 h2 = *reinterpret_cast<const uint2*>(ring + (size_t)((start - 1) & 3) * C);
    const uint2 x = *reinterpret_cast<const uint2*>(qkv + (size_t)i * C + c0);
    const float hx0[4] = {bf16_lo(h0.x), bf16_hi(h0.x), bf16_lo(h0.y), bf16_hi(h0.y)};
    const float hx1[4] = {bf16_lo(h1.x), bf16_hi(h1.x), bf16_lo(h1.y), bf16_hi(h1.y)};
    const float hx2[4] = {bf16_lo(h2.x), bf16_hi(h2.x), bf16_lo(h2.y), bf16_hi(h2.y)};
    const float xx[4] = {bf16_lo(x.x), bf16_hi(x.x), bf16_lo(x.y), bf16_hi(x.y)};
#pragma unroll
    for (int e = 0; e < 4; ++e) val[e] = conv_silu(conv_w, c0 + e, hx0[e], hx1[e], hx2[e], xx[e]);
    *reinterpret_cast<uint2*>(ring + (size_t)(start & 3) * C) = x;
  }
  if (blk >= 2 * Hk) {  // a value head: v and this row's gates
    const int h = blk - 2 * Hk;
    *reinterpret_cast<uint2*>(v_out + ((size_t)i * Hv + h) * kHead + 4 * lane) =
        make_uint2(pack_bf16x2(val[0], val[1]), pack_bf16x2(val[2], val[3]));
    if (lane == 0) {
      const size_t e = (size_t)i * Hv + h;
      float g, beta;
      make_gates(bf16_to_f(a_in[e]), bf16_to_f(b_in[e]), a_log[h], dt_bias[h], g, beta);
      g_out[e] = g;
      beta_out[e] = beta;
    }
    return;
  }
  const float m =
      warp_sum(val[0] * val[0] + val[1] * val[1] + val[2] * val[2] + val[3] * val[3]) *
      (1.f / kHead);
  const bool is_q = blk < Hk;
  const int head = is_q ? blk : blk - Hk;
  const float scale = is_q ? bfr(1.f / kHead) : bfr(0.08838834764831845f);
  const float rn = 1.f / sqrtf(m + 1e-6f);
  float o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e] = bf16_to_f(f_to_bf16(bfr(val[e] * rn) * scale));
  *reinterpret_cast<uint2*>((is_q ? q_out : k_out) + ((size_t)i * Hk + head) * kHead + 4 * lane) =
      make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
}

// Launches the decode-batch front: the vectorised kernel when every operand it
// reads or writes as 8-byte vectors is 8-byte aligned, else the per-channel one.
cudaError_t launch_decode_front(const uint16_t* qkv, const uint16_t* a, const uint16_t* b,
                                const uint16_t* conv_w, const float* a_log,
                                const float* dt_bias, uint16_t* taps, const int32_t* seq_slot,
                                const int32_t* seq_start, uint16_t* q, uint16_t* k, uint16_t* v,
                                float* g, float* beta, int B, int Hk, int Hv, int num_slots,
                                cudaStream_t s) {
  const uintptr_t any = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(taps) |
                        reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(conv_w);
  if ((any & 7) == 0) {
    const long long items = (long long)B * (2 * Hk + Hv);
    return launch_pdl(gdn_decode_front_kernel, dim3((unsigned)((items + 3) / 4)), dim3(128), 0,
                      s, qkv, a, b, conv_w, a_log, dt_bias, taps, seq_slot, seq_start, q, k, v,
                      g, beta, B, Hk, Hv, num_slots, device_status_word());
  }
  dim3 grid((B + kTokTileDecode - 1) / kTokTileDecode, 2 * Hk + Hv);
  return launch_pdl(gdn_prefill_front_kernel<kTokTileDecode>, grid, dim3(128), 0, s, qkv, a, b,
                    conv_w, a_log, dt_bias, taps, (const int32_t*)nullptr, seq_slot, seq_start,
                    q, k, v, g, beta, B, B, Hk, Hv, num_slots, device_status_word());
}

// Ring rows of each prompt's last min(3, n) inputs. grid (nseq, ceil(C / 256)).
__global__ void gdn_taps_store_kernel(const uint16_t* __restrict__ qkv, uint16_t* __restrict__ taps,
                                      const int32_t* __restrict__ cu,
                                      const int32_t* __restrict__ seq_slot,
                                      const int32_t* __restrict__ seq_start, int C, int num_slots,
                                      unsigned int* status) {
  const int s = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int slot = seq_slot != nullptr ? seq_slot[s] : s, start = seq_start[s];
  if (slot < 0) return;  // an inactive row
  if (slot >= num_slots || start < 0) {
    if (c == 0) flag_device(status, DEV_BAD_INDEX);
    return;
  }
  const int first = cu != nullptr ? cu[s] : s;
  const int n = cu != nullptr ? cu[s + 1] - first : 1;
  uint16_t* ring = taps + (size_t)slot * kRing * C;
  for (int p = n - 3 < 0 ? 0 : n - 3; p < n; ++p)
    ring[(size_t)((start + p) & 3) * C + c] = qkv[(size_t)(first + p) * C + c];
}

// out = rms_norm(y, w, eps) * silu(z) per row of `width` (a multiple of 128): one warp per row.
__global__ void gated_rmsnorm_kernel(const uint16_t* __restrict__ y, const uint16_t* __restrict__ z,
                                     const uint16_t* __restrict__ w, float eps,
                                     uint16_t* __restrict__ out, long long rows, int width) {
  pdl_wait();
  pdl_trigger();
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint16_t* yr = y + row * width;
  const uint16_t* zr = z + row * width;
  float ss = 0.f;
  for (int c = 4 * lane; c < width; c += 128) {
    const uint2 p = *reinterpret_cast<const uint2*>(yr + c);
    const float a0 = bf16_lo(p.x), a1 = bf16_hi(p.x), a2 = bf16_lo(p.y), a3 = bf16_hi(p.y);
    ss += a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
  }
  const float rstd = 1.f / sqrtf(warp_sum(ss) / width + eps);
  for (int c = 4 * lane; c < width; c += 128) {
    const uint2 p = *reinterpret_cast<const uint2*>(yr + c);
    const uint2 zz = *reinterpret_cast<const uint2*>(zr + c);
    const uint2 ww = __ldg(reinterpret_cast<const uint2*>(w + c));
    const float yv[4] = {bf16_lo(p.x), bf16_hi(p.x), bf16_lo(p.y), bf16_hi(p.y)};
    const float zv[4] = {bf16_lo(zz.x), bf16_hi(zz.x), bf16_lo(zz.y), bf16_hi(zz.y)};
    const float wv[4] = {bf16_lo(ww.x), bf16_hi(ww.x), bf16_lo(ww.y), bf16_hi(ww.y)};
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) r[e] = bfr(yv[e] * rstd * wv[e]) * silu_bf(zv[e]);
    uint2 o;
    o.x = pack_bf16x2(r[0], r[1]);
    o.y = pack_bf16x2(r[2], r[3]);
    *reinterpret_cast<uint2*>(out + row * width + c) = o;
  }
}

int check_heads(const char* name, int Hk, int Hv) {
  SC_REQUIRE(Hk > 0 && Hv > 0 && Hv % Hk == 0, SC_ERR_INVALID,
             "%s: Hv=%d must be a positive multiple of Hk=%d", name, Hv, Hk);
  SC_REQUIRE((long long)(2 * Hk + Hv) * kHead < (1LL << 31), SC_ERR_INVALID,
             "%s: too many channels", name);
  return SC_OK;
}

}  // namespace
}  // namespace sc

extern "C" int sc_gdn_decode_fused(const sc_bf16* qkv, const sc_bf16* z, const sc_bf16* a,
                                   const sc_bf16* b, const sc_bf16* conv_w, const float* A_log,
                                   const float* dt_bias, const sc_bf16* norm_w, float eps,
                                   sc_bf16* taps, const int32_t* position, float* state,
                                   const int32_t* state_slot, sc_bf16* out, int B, int Hk, int Hv,
                                   int num_slots, void* stream) {
  using namespace sc;
  const char* name = "sc_gdn_decode_fused";
  if (int rc = check_heads(name, Hk, Hv)) return rc;
  SC_REQUIRE(qkv && z && a && b && conv_w && A_log && dt_bias && norm_w && taps && position &&
                 state && out,
             SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(B >= 0 && num_slots > 0 && (state_slot != nullptr || num_slots >= B), SC_ERR_INVALID,
             "%s: B=%d num_slots=%d", name, B, num_slots);
  SC_REQUIRE((long long)B * Hv < (1LL << 31), SC_ERR_INVALID, "%s: B*Hv too large", name);
  SC_REQUIRE(eps >= 0.f, SC_ERR_INVALID, "%s: eps=%g", name, (double)eps);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(conv_w) & 7) == 0, SC_ERR_INVALID,
             "%s: conv_w must be 8-byte aligned", name);
  if (B == 0) return SC_OK;
  const int smem = kFChunks * kFChunkBytes + (int)sizeof(FusedSmem);
  static int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(gdn_decode_fused_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess)
      return set_error(SC_ERR_CUDA, "%s: smem attribute: %s", name, cudaGetErrorString(err));
    configured[dev] = 1;
  }
  dim3 grid(B * Hv, 2);
  gdn_decode_fused_kernel<<<grid, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      qkv, z, a, b, conv_w, A_log, dt_bias, norm_w, eps, taps, position, state, state_slot, out,
      Hk, Hv, num_slots, device_status_word());
  return check_launch(name);
}

extern "C" int sc_gdn_prefill_front(const sc_bf16* qkv, const sc_bf16* a, const sc_bf16* b,
                                    const sc_bf16* conv_w, const float* A_log,
                                    const float* dt_bias, sc_bf16* taps,
                                    const int32_t* cu_seqlens, const int32_t* seq_slot,
                                    const int32_t* seq_start, sc_bf16* q, sc_bf16* k, sc_bf16* v,
                                    float* g, float* beta, int nseq, int total_tokens, int Hk,
                                    int Hv, int num_slots, void* stream) {
  using namespace sc;
  const char* name = "sc_gdn_prefill_front";
  if (int rc = check_heads(name, Hk, Hv)) return rc;
  SC_REQUIRE(qkv && a && b && conv_w && A_log && dt_bias && taps && seq_start && q && k && v &&
                 g && beta,
             SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(nseq > 0 && total_tokens >= 0 && num_slots > 0, SC_ERR_INVALID,
             "%s: nseq=%d total_tokens=%d num_slots=%d", name, nseq, total_tokens, num_slots);
  SC_REQUIRE(cu_seqlens != nullptr || nseq == total_tokens, SC_ERR_INVALID,
             "%s: without cu_seqlens every sequence is one token (nseq=%d, tokens=%d)", name,
             nseq, total_tokens);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(conv_w) & 7) == 0, SC_ERR_INVALID,
             "%s: conv_w must be 8-byte aligned", name);
  if (total_tokens == 0) return SC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cu_seqlens == nullptr) {
    launch_decode_front(qkv, a, b, conv_w, A_log, dt_bias, taps, seq_slot, seq_start, q, k, v,
                        g, beta, total_tokens, Hk, Hv, num_slots, s);
  } else {
    dim3 grid((total_tokens + kTokTile - 1) / kTokTile, 2 * Hk + Hv);
    launch_pdl(gdn_prefill_front_kernel<kTokTile>, grid, dim3(128), 0, s, qkv, a, b, conv_w,
               A_log, dt_bias, taps, cu_seqlens, seq_slot, seq_start, q, k, v, g, beta, nseq,
               total_tokens, Hk, Hv, num_slots, device_status_word());
  }
  return check_launch(name);
}

extern "C" int sc_gdn_taps_store(const sc_bf16* qkv, sc_bf16* taps, const int32_t* cu_seqlens,
                                 const int32_t* seq_slot, const int32_t* seq_start, int nseq,
                                 int channels, int num_slots, void* stream) {
  using namespace sc;
  const char* name = "sc_gdn_taps_store";
  SC_REQUIRE(qkv && taps && seq_start, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(nseq >= 0 && channels > 0 && num_slots > 0, SC_ERR_INVALID,
             "%s: nseq=%d channels=%d num_slots=%d", name, nseq, channels, num_slots);
  if (nseq == 0) return SC_OK;
  dim3 grid(nseq, (channels + 255) / 256);
  gdn_taps_store_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qkv, taps, cu_seqlens, seq_slot, seq_start, channels, num_slots, device_status_word());
  return check_launch(name);
}

extern "C" int sc_gdn_sampler_gates(const sc_bf16* a, const sc_bf16* b, const float* a_log,
                                    const float* dt_bias, float* g, float* beta, int64_t rows,
                                    int Hv, void* stream) {
  using namespace sc;
  const char* name = "sc_gdn_sampler_gates";
  SC_REQUIRE(a && b && a_log && dt_bias && g && beta, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(rows >= 0 && Hv > 0 && rows <= (int64_t)1 << 40, SC_ERR_INVALID,
             "%s: rows=%lld Hv=%d", name, (long long)rows, Hv);
  const long long n = (long long)rows * Hv;
  if (n == 0) return SC_OK;
  const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 16);
  launch_pdl(sampler_gates_kernel, dim3((unsigned)blocks), dim3(256), 0,
             static_cast<cudaStream_t>(stream), reinterpret_cast<const uint16_t*>(a),
             reinterpret_cast<const uint16_t*>(b), a_log, dt_bias, g, beta, n, Hv);
  return check_launch(name);
}

extern "C" int sc_gated_rmsnorm(const sc_bf16* y, const sc_bf16* z, const sc_bf16* w, float eps,
                                sc_bf16* out, long long rows, int width, void* stream) {
  using namespace sc;
  const char* name = "sc_gated_rmsnorm";
  SC_REQUIRE(y && z && w && out, SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(rows >= 0 && width > 0 && width % 128 == 0, SC_ERR_INVALID,
             "%s: rows=%lld width=%d (a multiple of 128)", name, rows, width);
  SC_REQUIRE(((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(z) |
               reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 7) == 0,
             SC_ERR_INVALID, "%s: pointers must be 8-byte aligned", name);
  if (rows == 0) return SC_OK;
  const long long blocks = (rows + 7) / 8;
  launch_pdl(gated_rmsnorm_kernel, dim3((unsigned)blocks), dim3(256), 0,
             static_cast<cudaStream_t>(stream), y, z, w, eps, out, rows, width);
  return check_launch(name);
}

namespace {
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
}  // namespace

extern "C" size_t sc_gdn_decode_glue_workspace(int B, int Hk, int Hv) {
  if (B <= 0 || Hk <= 0 || Hv <= 0) return 0;
  const size_t qk = align256((size_t)B * Hk * 128 * 2), vy = align256((size_t)B * Hv * 128 * 2);
  const size_t gb = align256((size_t)B * Hv * 4);
  return 2 * qk + 2 * vy + 2 * gb;
}

extern "C" int sc_gdn_decode_glue(const sc_bf16* qkv, const sc_bf16* z, const sc_bf16* a,
                                  const sc_bf16* b, const sc_bf16* conv_w, const float* A_log,
                                  const float* dt_bias, const sc_bf16* norm_w, float eps,
                                  sc_bf16* taps, const int32_t* position, float* state,
                                  const int32_t* state_slot, sc_bf16* out, void* workspace,
                                  size_t workspace_bytes, int B, int Hk, int Hv, int num_slots,
                                  void* stream) {
  using namespace sc;
  const char* name = "sc_gdn_decode_glue";
  if (int rc = check_heads(name, Hk, Hv)) return rc;
  SC_REQUIRE(qkv && z && a && b && conv_w && A_log && dt_bias && norm_w && taps && position &&
                 state && out && workspace,
             SC_ERR_INVALID, "%s: null pointer", name);
  SC_REQUIRE(B >= 0 && num_slots > 0 && (state_slot != nullptr || num_slots >= B), SC_ERR_INVALID,
             "%s: B=%d num_slots=%d", name, B, num_slots);
  SC_REQUIRE(eps >= 0.f, SC_ERR_INVALID, "%s: eps=%g", name, (double)eps);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(conv_w) & 7) == 0 &&
                 ((reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(norm_w) |
                   reinterpret_cast<uintptr_t>(out)) & 7) == 0,
             SC_ERR_INVALID, "%s: conv_w, z, norm_w and out must be 8-byte aligned", name);
  SC_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, SC_ERR_INVALID,
             "%s: workspace must be 256-byte aligned", name);
  if (B == 0) return SC_OK;
  const size_t need = sc_gdn_decode_glue_workspace(B, Hk, Hv);
  SC_REQUIRE(workspace_bytes >= need, SC_ERR_INVALID, "%s: workspace %zu bytes < %zu", name,
             workspace_bytes, need);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  const size_t qk = align256((size_t)B * Hk * 128 * 2), vy = align256((size_t)B * Hv * 128 * 2);
  const size_t gb = align256((size_t)B * Hv * 4);
  uint16_t* q = reinterpret_cast<uint16_t*>(w);
  uint16_t* k = reinterpret_cast<uint16_t*>(w + qk);
  uint16_t* v = reinterpret_cast<uint16_t*>(w + 2 * qk);
  uint16_t* y = reinterpret_cast<uint16_t*>(w + 2 * qk + vy);
  float* g = reinterpret_cast<float*>(w + 2 * qk + 2 * vy);
  float* beta = reinterpret_cast<float*>(w + 2 * qk + 2 * vy + gb);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  launch_decode_front(qkv, a, b, conv_w, A_log, dt_bias, taps, state_slot, position, q, k, v, g,
                      beta, B, Hk, Hv, num_slots, s);
  if (int rc = check_launch(name)) return rc;
  if (int rc = gdn_bulk_launch(name, q, k, v, g, beta, state, state_slot, y, B, Hk, Hv, 128,
                               num_slots, s, BulkLaunch::kStateAhead))
    return rc;
  const long long rows = (long long)B * Hv;
  launch_pdl(gated_rmsnorm_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, s,
             (const uint16_t*)y, z, norm_w, eps, out, rows, 128);
  return check_launch(name);
}
