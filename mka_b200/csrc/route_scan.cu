// Stage 1 of the FastMKA forward: routing gate + causal prefix EMA + route blend.
//
//   lam[b,t,:] = softmax(logits[b,t,:] + b2)                  (router output)
//   L2[b,t,:]  = beta * L2[b,t-1,:] + (1 - beta) * X[b,t,:],  L2[b,-1,:] = 0
//   H[b,t,:]   = lam0 * X + lam1 * L2 (+ lam2 * L3[b, min(t, T3-1), :])
//
// Reference: causal_prefix_ema (mka/layers/session_memory.py:6-22),
// repeat_retrieval_to_length (session_memory.py:25-39), gate and blend
// (mka/layers/fastmka.py:91-96, mka/hf/attention.py:104-107). The reference
// runs the EMA as a Python loop of T steps (about 4T kernel launches); here the
// whole stage is one single-pass kernel that reads X (and L3) once and writes H
// once.
//
// Parallel scan. The EMA is a linear recurrence, so the state after a chunk is
// the chunk's zero-state scan ("aggregate") plus beta^len times the state that
// entered it; a chunk only needs its incoming state S_in to finish. Each CTA
// owns (batch row, 256-channel slice, 64-token chunk). Eight warps each scan
// eight tokens with 128-bit loads (lane = 8 channels); warp aggregates are
// combined in shared memory (two float4 planes per row, conflict-free). The
// chunk's incoming state comes from the preceding chunks of the same (batch,
// slice):
//   * short memory (beta^(64 k) < 2^-40 within k <= 32 chunks, e.g. beta = 0.9:
//     k = 5): the weighted sum of the k preceding chunk aggregates, read by k
//     warps in parallel. Older chunks weigh less than 2^-40 and are left out;
//     no chunk waits on more than the aggregates of its k predecessors;
//   * long memory: a decoupled look-back, each CTA publishing its aggregate,
//     then walking back over published aggregates until it finds a published
//     inclusive state.
// Chunk order comes from an atomic ticket, so a CTA only ever waits on CTAs
// that started before it. Waits are bounded; a timeout sets a status bit and the
// scan continues with a zero contribution. Three CTAs share an SM so that one
// CTA's waits are covered by the others' loads.
//
// Four kernels. route_ema_blend_kernel covers every mode (H or K/V output, a
// given L2, a carried EMA state, long memory). kv_window_kernel is the layer's
// case (K/V output, short memory, no carried state): a streaming kernel with
// no communication between CTAs (each CTA recomputes the state entering its
// token segment from a warm-up window). kv_small_kernel is the same case for
// inputs of at most 32 tokens (a decode step: 6.5 us against 16.8 us for 64
// sequences of one token): a warp per (batch row, slice) scans the tokens in
// order. kv_scan_kernel is the chunk-parallel look-back form, kept for tensors
// that do not suit TMA.
// Measured on the layer's K/V-mode scan (batch 4 x 8192 tokens, 1024
// channels, device time): 0.121 ms with a [32][8] shared-memory layout, whose
// eight-way bank conflicts kept the L1 pipe 74 % busy; 0.071-0.074 ms for the
// general kernel with the float4 planes; 0.057 ms for kv_scan_kernel; 0.040 ms
// for kv_window_kernel.
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

#ifndef FMKA_SCAN_WARPS
#define FMKA_SCAN_WARPS 8
#endif
constexpr int kWarps = FMKA_SCAN_WARPS;
constexpr int kTokPerWarp = 8;
constexpr int kChunkT = kWarps * kTokPerWarp;  // tokens per CTA (64)
constexpr int kSlice = 256;   // channels per CTA (32 lanes x 8)
constexpr int kThreads = kWarps * 32;

#ifndef FMKA_SCAN_MINB
#define FMKA_SCAN_MINB 3
#endif
// kv_scan_kernel: prefetch the RoPE table rows into L1 before the look-back
// (0.0588-0.0596 -> 0.0567-0.0571 ms on the layer's scan, same box).
#ifndef FMKA_SCAN_ROPE_PREFETCH
#define FMKA_SCAN_ROPE_PREFETCH 1
#endif
constexpr uint32_t kFlagAgg = 1;
constexpr uint32_t kFlagInc = 2;

struct ScanParams {
  const __nv_bfloat16* x;  // [B, T, D]
  int64_t x_sb, x_st;
  const float* logits;     // [B*T, L] router logits without the output bias
  const float* b2;         // [L] or null
  const float* gate;       // alternatively: precomputed gate [B*T, L] (logits == null)
  int L;
  const __nv_bfloat16* l2; // given L2 [B, T, D] (blend only, no scan) or null
  int64_t l2_sb, l2_st;
  const __nv_bfloat16* l3; // [B, T3, D] or null
  int64_t l3_sb, l3_st;
  int T3;
  float beta, one_minus_beta, beta8, beta_chunk;  // beta_chunk = beta^kChunkT
  // Short-memory look-back: when beta^(kChunkT * lb_max) < 2^-40 (beta <= ~0.98
  // at 128-token chunks), the state entering a chunk is the sum of the lb_max
  // preceding chunk aggregates weighted by beta^(kChunkT k); older chunks weigh less than 2^-40 of
  // the newest one, far below fp32 resolution, and are left out. Each chunk then
  // waits only for the aggregates of its lb_max predecessors (no inclusive
  // states, no chain). lb_max == 0: the full decoupled look-back.
  int lb_max;
  int B, T, D;
  __nv_bfloat16* h;        // [B, T, D]
  int64_t h_sb, h_st;
  float* lam;              // [B, T, L] or null
  // K/V mode (kv_k != null): the input is Y = X [Wk ; Wv]^T ([B, T, D] with
  // D = 2 * Hkv * 128), and the blend of Y and its EMA, plus kv_bias, with
  // rotate-half RoPE on the K half, is stored head-split into kv_k / kv_v
  // ([B, Hkv, Tcap, 128], strides kv_sb, kv_sh, kv_st) at token slot t + t_offset.
  __nv_bfloat16* kv_k;
  __nv_bfloat16* kv_v;
  int64_t kv_sb, kv_sh, kv_st;
  int t_offset;
  const float* kv_bias;    // [D] or null
  const float* rope_cos;   // [*, T, 128] fp32 or null
  const float* rope_sin;
  int64_t rope_sb, rope_st;
  const float* ema_init;   // [B, D] fp32 EMA state before token 0 (null: zero), scan mode only
  float* ema_final;        // [B, D] fp32 EMA state after token T-1 (null: not written)
  uint32_t* ticket;
  uint32_t* flags;         // [nseq * nchunks]
  float* agg;              // [nseq * nchunks * kSlice]
  float* inc;              // [nseq * nchunks * kSlice]
  int nds, nchunks;
  uint32_t* status;
  // kv_window_kernel: tokens of the warm-up window; the CTAs of slices with K
  // heads (ds < nds_k, the first n_ctas_k CTAs) and of V-only slices have their
  // own segment lengths; whether the L3 / RoPE tensor maps have a batch dimension
  int win_tokens, seg_len_k, seg_len_v, nds_k, n_ctas_k;
  int l3_bcast, rope_bcast;
  float beta4, beta32;  // kv_window_kernel: beta^(tokens per consumer warp), beta^(tokens per sub-chunk)
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  f[0] = bf16lo_to_f32(u.x);
  f[1] = bf16hi_to_f32(u.x);
  f[2] = bf16lo_to_f32(u.y);
  f[3] = bf16hi_to_f32(u.y);
  f[4] = bf16lo_to_f32(u.z);
  f[5] = bf16hi_to_f32(u.z);
  f[6] = bf16lo_to_f32(u.w);
  f[7] = bf16hi_to_f32(u.w);
}

__device__ __forceinline__ float ipow(float b, int e);

// A lane's 8 channels in shared memory as two float4 planes ([2][32] per row):
// consecutive lanes hit consecutive 16-byte words, so a warp's access is
// conflict-free (a [32][8] float layout would serialise it eight ways).
__device__ __forceinline__ void put8(float4 (&row)[2][32], int lane, const float (&v)[8]) {
  row[0][lane] = make_float4(v[0], v[1], v[2], v[3]);
  row[1][lane] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void get8(const float4 (&row)[2][32], int lane, float (&v)[8]) {
  const float4 a = row[0][lane], b = row[1][lane];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Warp 0 of the CTA that owns (seq, chunk): publishes the chunk aggregate `a`
// (state after the chunk from a zero state, this lane's 8 channels), finds the
// state entering the chunk by the decoupled look-back, publishes the chunk's
// inclusive state and returns the incoming state in sin_.
__device__ __forceinline__ void chunk_lookback(const ScanParams& p, int seq, int chunk, const float (&a)[8],
                                               float (&sin_)[8]) {
  const int lane = lane_id();
  // Publishing: every lane stores its 8 channels, __syncwarp orders those stores
  // before lane 0's release store of the flag (the release is cumulative over
  // them), so no separate fence is needed.
  const int64_t rec = (int64_t)seq * p.nchunks + chunk;
#pragma unroll
  for (int c = 0; c < 8; ++c) sin_[c] = 0.f;
  if (chunk == 0) {
    float4* dst = reinterpret_cast<float4*>(p.inc + rec * kSlice + lane * 8);
    __stcg(dst, make_float4(a[0], a[1], a[2], a[3]));
    __stcg(dst + 1, make_float4(a[4], a[5], a[6], a[7]));
    __syncwarp();
    if (lane == 0) st_release_u32(p.flags + rec, kFlagInc);
  } else {
    {
      float4* dst = reinterpret_cast<float4*>(p.agg + rec * kSlice + lane * 8);
      __stcg(dst, make_float4(a[0], a[1], a[2], a[3]));
      __stcg(dst + 1, make_float4(a[4], a[5], a[6], a[7]));
      __syncwarp();
      if (lane == 0) st_release_u32(p.flags + rec, kFlagAgg);
    }
    // Parallel look-back: lane l watches predecessor chunk (base - l); one
    // round trip finds the nearest predecessor whose inclusive state is
    // published (chunk -1 counts as an inclusive zero state), then the
    // aggregates in between and that inclusive state are read together.
    const uint32_t* seq_flags = p.flags + (int64_t)seq * p.nchunks;
    const int64_t seq_rec = (int64_t)seq * p.nchunks;
    int base = chunk - 1;  // nearest predecessor not yet accounted for
    float mult = 1.f;      // beta^(kChunkT * (chunk - 1 - base))
    const uint64_t tstart = globaltimer_ns();
    while (true) {
      const int pc = base - lane;
      const uint32_t f = pc >= 0 ? ld_acquire_u32(seq_flags + pc) : kFlagInc;
      const uint32_t inc_mask = __ballot_sync(0xffffffffu, f == kFlagInc);
      const uint32_t nil_mask = __ballot_sync(0xffffffffu, f == 0u);
      const int l_inc = inc_mask ? __ffs(inc_mask) - 1 : 32;
      const uint32_t needed = l_inc >= 32 ? 0xffffffffu : ((1u << l_inc) - 1u);
      if (nil_mask & needed) {  // an aggregate on the way is not published yet
        if (globaltimer_ns() - tstart > kWaitLimitNs) {
          if (lane == 0) atomicOr(p.status, kStatusLookbackTimeout);
          break;  // give up: the rest counts as zero
        }
        __nanosleep(32);
        continue;
      }
      __syncwarp();  // orders the lanes' acquires before every lane's record reads
      const int nk = l_inc >= 32 ? 32 : l_inc + 1;
      for (int k = 0; k < nk; ++k) {
        const int pck = base - k;
        if (pck < 0) break;  // the zero state before the sequence
        const float* src = (k == l_inc ? p.inc : p.agg) + (seq_rec + pck) * kSlice + lane * 8;
        const float4 v0 = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 v1 = __ldcg(reinterpret_cast<const float4*>(src) + 1);
        sin_[0] += mult * v0.x;
        sin_[1] += mult * v0.y;
        sin_[2] += mult * v0.z;
        sin_[3] += mult * v0.w;
        sin_[4] += mult * v1.x;
        sin_[5] += mult * v1.y;
        sin_[6] += mult * v1.z;
        sin_[7] += mult * v1.w;
        mult *= p.beta_chunk;
      }
      if (l_inc < 32) break;
      base -= 32;
    }
    float inc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) inc[c] = a[c] + p.beta_chunk * sin_[c];
    float4* dst = reinterpret_cast<float4*>(p.inc + rec * kSlice + lane * 8);
    __stcg(dst, make_float4(inc[0], inc[1], inc[2], inc[3]));
    __stcg(dst + 1, make_float4(inc[4], inc[5], inc[6], inc[7]));
    __syncwarp();
    if (lane == 0) st_release_u32(p.flags + rec, kFlagInc);
  }
}

// Short-memory look-back, run by every warp: warp w adds the aggregates of
// predecessor chunks chunk-1-k, k = w, w + kWarps, ... < lb_max, each weighted
// by beta^(kChunkT k), into part (this lane's 8 channels). Every lane polls the flag
// (a broadcast load) so that each lane's own acquire orders its record reads.
__device__ __forceinline__ void short_lookback(const ScanParams& p, int seq, int chunk, int warp, float (&part)[8]) {
  const int lane = lane_id();
  const uint32_t* seq_flags = p.flags + (int64_t)seq * p.nchunks;
  const int64_t seq_rec = (int64_t)seq * p.nchunks;
#pragma unroll
  for (int c = 0; c < 8; ++c) part[c] = 0.f;
  for (int k = warp; k < p.lb_max; k += kWarps) {
    const int pc = chunk - 1 - k;
    if (pc < 0) break;
    const uint64_t tstart = globaltimer_ns();
    bool ok = true;
    while (ld_acquire_u32(seq_flags + pc) == 0u) {
      if (globaltimer_ns() - tstart > kWaitLimitNs) {
        if (lane == 0) atomicOr(p.status, kStatusLookbackTimeout);
        ok = false;  // give up: this predecessor counts as zero
        break;
      }
      __nanosleep(32);
    }
    if (!ok) continue;
    const float w = ipow(p.beta_chunk, k);
    const float* src = p.agg + (seq_rec + pc) * kSlice + lane * 8;
    const float4 v0 = __ldcg(reinterpret_cast<const float4*>(src));
    const float4 v1 = __ldcg(reinterpret_cast<const float4*>(src) + 1);
    part[0] += w * v0.x;
    part[1] += w * v0.y;
    part[2] += w * v0.z;
    part[3] += w * v0.w;
    part[4] += w * v1.x;
    part[5] += w * v1.y;
    part[6] += w * v1.z;
    part[7] += w * v1.w;
  }
}

// b^e for an integer e >= 0 by repeated squaring (exact in sign for b < 0,
// which exp2(e * log2 b) is not).
__device__ __forceinline__ float ipow(float b, int e) {
  float r = 1.f;
  while (e > 0) {
    if (e & 1) r *= b;
    b *= b;
    e >>= 1;
  }
  return r;
}

__global__ void __launch_bounds__(kThreads, FMKA_SCAN_MINB) route_ema_blend_kernel(const __grid_constant__ ScanParams p) {
  __shared__ uint32_t s_tile;
  __shared__ float4 s_wagg[kWarps][2][32];  // each warp's zero-state aggregate (put8 / get8 layout)
  __shared__ float4 s_in[2][32];            // full look-back: the state entering the chunk
  __shared__ float4 s_part[kWarps][2][32];  // short look-back: each warp's weighted predecessor sum
  __shared__ float s_lam[kChunkT][4];

  const int warp = warp_id();
  const int lane = lane_id();

  const bool scan = p.l2 == nullptr;  // grid-uniform
  if (threadIdx.x == 0) s_tile = scan ? atomicAdd(p.ticket, 1u) : blockIdx.x;
  __syncthreads();
  const int tile = static_cast<int>(s_tile);
  const int nseq = p.B * p.nds;
  const int chunk = tile / nseq;
  const int seq = tile % nseq;
  const int b = seq / p.nds;
  const int ds = seq % p.nds;
  const int t0 = chunk * kChunkT;
  const int d0 = ds * kSlice + lane * 8;
  const bool ch_ok = d0 < p.D;

  // ---- gate for the chunk's tokens ----
  if (threadIdx.x < kChunkT) {
    const int t = t0 + threadIdx.x;
    float g[4] = {0.f, 0.f, 0.f, 0.f};
    if (t < p.T) {
      const int64_t row = (int64_t)b * p.T + t;
      if (p.logits != nullptr) {
        float mx = -INFINITY;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
          if (l < p.L) {
            g[l] = p.logits[row * p.L + l] + (p.b2 ? p.b2[l] : 0.f);
            mx = fmaxf(mx, g[l]);
          }
        }
        float sum = 0.f;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
          if (l < p.L) {
            g[l] = __expf(g[l] - mx);
            sum += g[l];
          }
        }
        const float inv = 1.f / sum;
#pragma unroll
        for (int l = 0; l < 4; ++l) g[l] *= inv;
      } else {
#pragma unroll
        for (int l = 0; l < 4; ++l)
          if (l < p.L) g[l] = p.gate[row * p.L + l];
      }
      if (p.lam != nullptr && ds == 0) {
#pragma unroll
        for (int l = 0; l < 4; ++l)
          if (l < p.L) p.lam[row * p.L + l] = g[l];
      }
    }
#pragma unroll
    for (int l = 0; l < 4; ++l) s_lam[threadIdx.x][l] = g[l];
  }

  // ---- load this warp's 8 tokens x 8 channels (128-bit loads) ----
  const int tw = t0 + warp * kTokPerWarp;
  uint4 xr[kTokPerWarp];
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i) {
    const int t = tw + i;
    if (ch_ok && t < p.T) {
      xr[i] = __ldcs(reinterpret_cast<const uint4*>(p.x + (int64_t)b * p.x_sb + (int64_t)t * p.x_st + d0));
    } else {
      xr[i] = make_uint4(0, 0, 0, 0);
    }
  }

  // ---- local scan from a zero state: only the warp aggregate is kept; the
  // output pass re-runs the recurrence from the true incoming state ----
  if (scan) {
    float st[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kTokPerWarp; ++i) {
      float xf[8];
      unpack8(xr[i], xf);
#pragma unroll
      for (int c = 0; c < 8; ++c) st[c] = p.beta * st[c] + p.one_minus_beta * xf[c];
    }
    put8(s_wagg[warp], lane, st);
  }
  __syncthreads();

  // ---- chunk aggregate + look-back ----
  const bool short_lb = p.lb_max > 0;  // grid-uniform
  if (scan && short_lb) {
    if (warp == 0) {
      // publish this chunk's aggregate before waiting on anything
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        float wa[8];
        get8(s_wagg[w], lane, wa);
#pragma unroll
        for (int c = 0; c < 8; ++c) a[c] = p.beta8 * a[c] + wa[c];
      }
      const int64_t rec = (int64_t)seq * p.nchunks + chunk;
      float4* dst = reinterpret_cast<float4*>(p.agg + rec * kSlice + lane * 8);
      __stcg(dst, make_float4(a[0], a[1], a[2], a[3]));
      __stcg(dst + 1, make_float4(a[4], a[5], a[6], a[7]));
      __syncwarp();
      if (lane == 0) st_release_u32(p.flags + rec, kFlagAgg);
    }
    if (warp < p.lb_max) {
      float part[8];
      short_lookback(p, seq, chunk, warp, part);
      put8(s_part[warp], lane, part);
    }
  } else if (scan && warp == 0) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      float wa[8];
      get8(s_wagg[w], lane, wa);
#pragma unroll
      for (int c = 0; c < 8; ++c) a[c] = p.beta8 * a[c] + wa[c];
    }
    float sin_[8];
    chunk_lookback(p, seq, chunk, a, sin_);
    put8(s_in, lane, sin_);
  }
  __syncthreads();

  // ---- state entering this warp's tokens ----
  float st[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (scan) {
    if (short_lb) {
      const int nparts = p.lb_max < kWarps ? p.lb_max : kWarps;
      for (int w = 0; w < nparts; ++w) {
        float v[8];
        get8(s_part[w], lane, v);
#pragma unroll
        for (int c = 0; c < 8; ++c) st[c] += v[c];
      }
    } else {
      get8(s_in, lane, st);
    }
    for (int w = 0; w < warp; ++w) {
      float v[8];
      get8(s_wagg[w], lane, v);
#pragma unroll
      for (int c = 0; c < 8; ++c) st[c] = p.beta8 * st[c] + v[c];
    }
    if (p.ema_init != nullptr && ch_ok) {
      // the scan runs from a zero state; a state s before token 0 adds
      // beta^t * s to the state entering token t
      const float dec = ipow(p.beta, tw);
      const float4 i0 = *reinterpret_cast<const float4*>(p.ema_init + (int64_t)b * p.D + d0);
      const float4 i1 = *reinterpret_cast<const float4*>(p.ema_init + (int64_t)b * p.D + d0 + 4);
      st[0] += dec * i0.x;
      st[1] += dec * i0.y;
      st[2] += dec * i0.z;
      st[3] += dec * i0.w;
      st[4] += dec * i1.x;
      st[5] += dec * i1.y;
      st[6] += dec * i1.z;
      st[7] += dec * i1.w;
    }
  }

  // ---- blend and store ----
  float kvb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // K/V bias of this lane's channels, loaded once
  if (p.kv_k != nullptr && p.kv_bias != nullptr && ch_ok) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + d0));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + d0 + 4));
    kvb[0] = b0.x; kvb[1] = b0.y; kvb[2] = b0.z; kvb[3] = b0.w;
    kvb[4] = b1.x; kvb[5] = b1.y; kvb[6] = b1.z; kvb[7] = b1.w;
  }
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i) {
    const int t = tw + i;
    const int tl = warp * kTokPerWarp + i;
    const float g0 = s_lam[tl][0], g1 = s_lam[tl][1], g2 = s_lam[tl][2];
    float xf[8];
    unpack8(xr[i], xf);
    float l3f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (p.l3 != nullptr && ch_ok && t < p.T) {
      const int t3 = t < p.T3 ? t : p.T3 - 1;
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p.l3 + (int64_t)b * p.l3_sb + (int64_t)t3 * p.l3_st + d0));
      unpack8(u, l3f);
    }
    float l2f[8];
    if (!scan && ch_ok && t < p.T) {
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p.l2 + (int64_t)b * p.l2_sb + (int64_t)t * p.l2_st + d0));
      unpack8(u, l2f);
    }
    float o[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (scan) {
        st[c] = p.beta * st[c] + p.one_minus_beta * xf[c];  // L2 at token t
      } else {
        st[c] = (ch_ok && t < p.T) ? l2f[c] : 0.f;
      }
      float v = g0 * xf[c] + g1 * st[c];
      if (p.l3 != nullptr) v += g2 * l3f[c];
      o[c] = v;
    }
    if (scan && p.ema_final != nullptr && ch_ok && t == p.T - 1) {
      float* f = p.ema_final + (int64_t)b * p.D + d0;
      *reinterpret_cast<float4*>(f) = make_float4(st[0], st[1], st[2], st[3]);
      *reinterpret_cast<float4*>(f + 4) = make_float4(st[4], st[5], st[6], st[7]);
    }
    if (p.kv_k != nullptr) {
      // K/V of the blend: bias, then RoPE on the K half. Channel d0 + c of a
      // 128-dim head pairs with d0 + c -/+ 64, which lives 8 lanes away.
      const int nk = p.D >> 1;  // K channels
      const bool is_k = d0 < nk;
#pragma unroll
      for (int c = 0; c < 8; ++c) o[c] += kvb[c];
      const int dim = d0 & 127;  // position of this lane's 8 channels in their head
      if (p.rope_cos != nullptr) {
        float partner[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) partner[c] = __shfl_xor_sync(0xffffffffu, o[c], 8);
        if (is_k && ch_ok && t < p.T) {
          const int64_t roff = (int64_t)b * p.rope_sb + (int64_t)t * p.rope_st + dim;
          const float sign = dim < 64 ? -1.f : 1.f;  // rotate_half: (-x2, x1)
          const float4 c0 = *reinterpret_cast<const float4*>(p.rope_cos + roff);
          const float4 c1 = *reinterpret_cast<const float4*>(p.rope_cos + roff + 4);
          const float4 s0 = *reinterpret_cast<const float4*>(p.rope_sin + roff);
          const float4 s1 = *reinterpret_cast<const float4*>(p.rope_sin + roff + 4);
          const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
          for (int c = 0; c < 8; ++c) o[c] = o[c] * cs[c] + sign * partner[c] * sn[c];
        }
      }
      if (ch_ok && t < p.T) {
        const int head = (is_k ? d0 : d0 - nk) >> 7;
        __nv_bfloat16* dst = (is_k ? p.kv_k : p.kv_v) + (int64_t)b * p.kv_sb + (int64_t)head * p.kv_sh +
                             (int64_t)(t + p.t_offset) * p.kv_st + dim;
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        *reinterpret_cast<uint4*>(dst) = w;
      }
    } else if (ch_ok && t < p.T) {
      uint4 w;
      w.x = pack_bf16x2(o[0], o[1]);
      w.y = pack_bf16x2(o[2], o[3]);
      w.z = pack_bf16x2(o[4], o[5]);
      w.w = pack_bf16x2(o[6], o[7]);
      __stcs(reinterpret_cast<uint4*>(p.h + (int64_t)b * p.h_sb + (int64_t)t * p.h_st + d0), w);
    }
  }
}


// ---------------------------------------------------------------------------
// The layer's stage 1 as a specialised kernel: K/V output, short look-back,
// no carried EMA state, whole 256-channel slices. The same chunking and
// look-back as route_ema_blend_kernel, with the mode decided at compile time
// (RoPE, bias, third level) and the state kept scaled: u_t = beta u_{t-1} + y_t,
// so that EMA_t = (1 - beta) u_t and each step is one FMA; the factor (1 - beta)
// moves into the gate (lam1 (1 - beta)) and the chunk aggregates and the
// look-back work in u units throughout. Base pointers are formed once per
// thread and advanced by their strides; only the stores of the last chunk's
// rows past T are predicated (those rows read row T - 1 and come after every
// valid token, so they change only an aggregate that no chunk reads).
template <bool kRope, bool kBias, bool kL3>
__global__ void __launch_bounds__(kThreads, FMKA_SCAN_MINB) kv_scan_kernel(const __grid_constant__ ScanParams p) {
  __shared__ uint32_t s_tile;
  __shared__ float4 s_wagg[kWarps][2][32];
  __shared__ float4 s_part[kWarps][2][32];
  __shared__ float4 s_gate[kChunkT];  // lam0, lam1 (1 - beta), lam2 per token

  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) s_tile = atomicAdd(p.ticket, 1u);
  __syncthreads();
  const int tile = static_cast<int>(s_tile);
  const int nseq = p.B * p.nds;
  const int chunk = tile / nseq;
  const int seq = tile % nseq;
  const int b = seq / p.nds;
  const int ds = seq % p.nds;
  const int T = p.T;
  const int t0 = chunk * kChunkT;
  const int tw = t0 + warp * kTokPerWarp;
  const int d0 = ds * kSlice + lane * 8;
  const float beta = p.beta;

  // ---- this warp's 8 rows x 8 channels per lane (read again, from L1, by
  // the blend, so that they are not held in registers across the look-back) ----
  const __nv_bfloat16* xw = p.x + (int64_t)b * p.x_sb + d0 + (int64_t)tw * p.x_st;
  const int last = T - 1 - tw;  // rows i > last repeat row T - 1
  uint4 xr[kTokPerWarp];
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i)
    xr[i] = __ldg(reinterpret_cast<const uint4*>(xw + (int64_t)(i < last ? i : last) * p.x_st));
#if FMKA_SCAN_ROPE_PREFETCH
  // ---- bring this warp's RoPE table rows into L1 now, so that the blend after
  // the look-back finds them there (8 tokens x cos, sin x 4 lines of 128 bytes) ----
  if (kRope && d0 < (p.D >> 1)) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int line = lane + 32 * j;
      const int t = tw + (line >> 3);
      if (t < T) {
        const float* row = ((line >> 2) & 1 ? p.rope_sin : p.rope_cos) + (int64_t)b * p.rope_sb + (int64_t)t * p.rope_st;
        asm volatile("prefetch.global.L1 [%0];" ::"l"(row + (line & 3) * 32));
      }
    }
  }
#endif
  // ---- gate of the chunk's tokens ----
  if (threadIdx.x < kChunkT) {
    const int t = t0 + threadIdx.x;
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < T) {
      const int64_t row = (int64_t)b * T + t;
      const float* lg = p.logits + row * p.L;
      float a0 = lg[0] + (p.b2 ? p.b2[0] : 0.f);
      float a1 = lg[1] + (p.b2 ? p.b2[1] : 0.f);
      float a2 = kL3 ? lg[2] + (p.b2 ? p.b2[2] : 0.f) : -INFINITY;
      const float mx = fmaxf(fmaxf(a0, a1), a2);
      a0 = __expf(a0 - mx);
      a1 = __expf(a1 - mx);
      a2 = kL3 ? __expf(a2 - mx) : 0.f;
      const float inv = 1.f / (a0 + a1 + a2);
      a0 *= inv;
      a1 *= inv;
      a2 *= inv;
      if (p.lam != nullptr && ds == 0) {
        p.lam[row * p.L] = a0;
        p.lam[row * p.L + 1] = a1;
        if (kL3) p.lam[row * p.L + 2] = a2;
      }
      g = make_float4(a0, a1 * p.one_minus_beta, a2, 0.f);
    }
    s_gate[threadIdx.x] = g;
  }

  // ---- zero-state scan of this warp's 8 tokens (u units) ----
  {
    float u[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kTokPerWarp; ++i) {
      float xf[8];
      unpack8(xr[i], xf);
#pragma unroll
      for (int c = 0; c < 8; ++c) u[c] = fmaf(beta, u[c], xf[c]);
    }
    put8(s_wagg[warp], lane, u);
  }
  __syncthreads();

  // ---- chunk aggregate, then the k preceding chunks' aggregates ----
  if (warp == 0) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      float wa[8];
      get8(s_wagg[w], lane, wa);
#pragma unroll
      for (int c = 0; c < 8; ++c) a[c] = fmaf(p.beta8, a[c], wa[c]);
    }
    const int64_t rec = (int64_t)seq * p.nchunks + chunk;
    float4* dst = reinterpret_cast<float4*>(p.agg + rec * kSlice + lane * 8);
    __stcg(dst, make_float4(a[0], a[1], a[2], a[3]));
    __stcg(dst + 1, make_float4(a[4], a[5], a[6], a[7]));
    __syncwarp();
    if (lane == 0) st_release_u32(p.flags + rec, kFlagAgg);
  }
  const int nparts = p.lb_max < kWarps ? p.lb_max : kWarps;
  if (warp < nparts) {
    float part[8];
    short_lookback(p, seq, chunk, warp, part);
    put8(s_part[warp], lane, part);
  }
  __syncthreads();

  // ---- state entering this warp's tokens ----
  float u[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < nparts; ++w) {
    float v[8];
    get8(s_part[w], lane, v);
#pragma unroll
    for (int c = 0; c < 8; ++c) u[c] += v[c];
  }
  for (int w = 0; w < warp; ++w) {
    float v[8];
    get8(s_wagg[w], lane, v);
#pragma unroll
    for (int c = 0; c < 8; ++c) u[c] = fmaf(p.beta8, u[c], v[c]);
  }

  // ---- blend, bias, RoPE, head-split store ----
  const int nk = p.D >> 1;
  const bool is_k = d0 < nk;
  const int dim = d0 & 127;
  const int head = (is_k ? d0 : d0 - nk) >> 7;
  __nv_bfloat16* dst = (is_k ? p.kv_k : p.kv_v) + (int64_t)b * p.kv_sb + (int64_t)head * p.kv_sh +
                       (int64_t)(tw + p.t_offset) * p.kv_st + dim;
  float kvb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (kBias) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + d0));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + d0 + 4));
    kvb[0] = b0.x; kvb[1] = b0.y; kvb[2] = b0.z; kvb[3] = b0.w;
    kvb[4] = b1.x; kvb[5] = b1.y; kvb[6] = b1.z; kvb[7] = b1.w;
  }
  const float* cosp = nullptr;
  const float* sinp = nullptr;
  uint32_t sign_flip = 0u;  // rotate_half: the first 64 dims take -x2 (sign bit flipped)
  if (kRope) {
    cosp = p.rope_cos + (int64_t)b * p.rope_sb + (int64_t)tw * p.rope_st + dim;
    sinp = p.rope_sin + (int64_t)b * p.rope_sb + (int64_t)tw * p.rope_st + dim;
    sign_flip = dim < 64 ? 0x80000000u : 0u;
  }
  const __nv_bfloat16* y3p = nullptr;
  if (kL3) y3p = p.l3 + (int64_t)b * p.l3_sb + d0;
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i) {
    const int t = tw + i;
    const float4 g = s_gate[warp * kTokPerWarp + i];
    float xf[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(xw + (int64_t)(i < last ? i : last) * p.x_st)), xf);
    float o[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      u[c] = fmaf(beta, u[c], xf[c]);
      o[c] = fmaf(g.x, xf[c], fmaf(g.y, u[c], kvb[c]));
    }
    if (kL3) {
      const int t3 = t < p.T3 ? t : p.T3 - 1;
      float y3f[8];
      unpack8(__ldcs(reinterpret_cast<const uint4*>(y3p + (int64_t)t3 * p.l3_st)), y3f);
#pragma unroll
      for (int c = 0; c < 8; ++c) o[c] = fmaf(g.z, y3f[c], o[c]);
    }
    if (kRope) {
      float partner[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) partner[c] = __shfl_xor_sync(0xffffffffu, o[c], 8);
      if (is_k && t < T) {
        const float4 c0 = __ldg(reinterpret_cast<const float4*>(cosp + (int64_t)i * p.rope_st));
        const float4 c1 = __ldg(reinterpret_cast<const float4*>(cosp + (int64_t)i * p.rope_st + 4));
        const float4 s0 = __ldg(reinterpret_cast<const float4*>(sinp + (int64_t)i * p.rope_st));
        const float4 s1 = __ldg(reinterpret_cast<const float4*>(sinp + (int64_t)i * p.rope_st + 4));
        const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c)
          o[c] = fmaf(__uint_as_float(__float_as_uint(partner[c]) ^ sign_flip), sn[c], o[c] * cs[c]);
      }
    }
    if (t < T) {
      uint4 w;
      w.x = pack_bf16x2(o[0], o[1]);
      w.y = pack_bf16x2(o[2], o[3]);
      w.z = pack_bf16x2(o[4], o[5]);
      w.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(dst + (int64_t)i * p.kv_st) = w;
    }
  }
}


// ---------------------------------------------------------------------------
// The layer's stage 1 as a streaming kernel: no communication between CTAs.
//
// With short memory (beta^W < 2^-40 for a window of W tokens) the state
// entering token s is, to within 2^-40 of its newest term, the zero-state scan
// of the W tokens before s. So each CTA owns a segment of tokens of one
// (batch row, 256-channel slice), first scans the W tokens before the segment
// (warm-up: loads and FMAs only) and then streams the segment, carrying the
// state from sub-chunk to sub-chunk. There is no look-back, no ticket and no
// flag memory; the grid is one CTA per SM.
//
// Warp roles: warp 8 drives a ring of shared-memory stages with TMA (per
// 32-token sub-chunk: the y tile [32 x 256] bf16, and in the segment proper the
// y3 tile and the RoPE cos / sin rows [32 x 128] fp32) and writes the gate of
// the sub-chunk's 32 tokens into the stage, from router logits it loaded one
// ring length earlier (lane i: token i); warps 0-7 take 4 tokens each. A lane
// holds channels 4q..4q+3 and 64+4q..64+4q+3 of one head (q = lane % 16, head
// = lane / 16 within the slice), so the rotate-half partner of every channel is
// in the same lane and the RoPE needs no shuffle. Per sub-chunk a warp scans its
// 4 tokens from a zero state, publishes the aggregate, and after one named
// barrier finds its incoming state from the carried state and the aggregates of
// the warps before it; warp 7 carries the state to the next sub-chunk. The
// state is kept in u units (u_t = beta u_{t-1} + y_t, EMA = (1 - beta) u).
// During the warm-up each warp keeps its own running sum of its aggregates
// (A_w = beta^32 A_w + a_w), which needs no barrier; the state at the segment
// start is sum_w beta^(4 (7 - w)) A_w.
// Tokens per consumer warp: 8 (64-token sub-chunks) halves the barriers and
// cross-warp combines per token against 4; measured on the layer's scan at
// batch 4 x 8192: 0.0339 ms against 0.0410 alone, 0.0397 against 0.0448 ms
// inside the step (batch 2: 0.0205 both).
#ifndef FMKA_WIN_TPW
#define FMKA_WIN_TPW 8
#endif
constexpr int kWinWarps = 8;                             // consumer warps
constexpr int kWinTpw = FMKA_WIN_TPW;                    // tokens per consumer warp
constexpr int kWinTok = kWinWarps * kWinTpw;             // tokens per sub-chunk
constexpr int kWinHalves = kWinTok / 32;                 // gates a producer lane writes per sub-chunk
constexpr int kWinThreads = (kWinWarps + 1) * 32;
constexpr int kWinRowBytes = kSlice * 2;                 // one token's 256 channels, bf16
constexpr int kWinYBytes = kWinTok * kWinRowBytes;       // 16 KB
constexpr int kWinRopeBytes = kWinTok * 128 * 4;         // 16 KB for cos, 16 KB for sin
constexpr int kWinGateBytes = kWinTok * 16;             // float4 gate per token
static_assert(kWinTpw == 4 || kWinTpw == 8, "4 or 8 tokens per consumer warp");
constexpr int kWinSmemBudget = 200 * 1024;
#ifndef FMKA_WIN_WARM_MULTI
#define FMKA_WIN_WARM_MULTI 1
#endif

template <bool kRope, bool kL3>
struct WinLayout {
  static constexpr int y = 0;
  static constexpr int y3 = kWinYBytes;
  static constexpr int cs = y3 + (kL3 ? kWinYBytes : 0);
  static constexpr int sn = cs + (kRope ? kWinRopeBytes : 0);
  static constexpr int gate = sn + (kRope ? kWinRopeBytes : 0);
  static constexpr int stage = gate + kWinGateBytes;
  static constexpr int fit = kWinSmemBudget / stage;
  static constexpr int stages = fit > 8 ? 8 : fit;
  static constexpr int bytes = stages * stage;
  // the warm-up needs only y: a stage then holds this many 32-token y tiles
  static constexpr int warm_tiles = FMKA_WIN_WARM_MULTI ? gate / kWinYBytes : 1;
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 4 bf16 at channels c..c+3 and 4 at c+64..c+67 -> 8 floats (lo then hi)
__device__ __forceinline__ void unpack_lohi(const uint2& lo, const uint2& hi, float (&f)[8]) {
  f[0] = bf16lo_to_f32(lo.x);
  f[1] = bf16hi_to_f32(lo.x);
  f[2] = bf16lo_to_f32(lo.y);
  f[3] = bf16hi_to_f32(lo.y);
  f[4] = bf16lo_to_f32(hi.x);
  f[5] = bf16hi_to_f32(hi.x);
  f[6] = bf16lo_to_f32(hi.y);
  f[7] = bf16hi_to_f32(hi.y);
}

template <bool kRope, bool kBias, bool kL3>
__global__ void __launch_bounds__(kWinThreads, 1)
    kv_window_kernel(const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmY3,
                     const __grid_constant__ CUtensorMap tmCos, const __grid_constant__ CUtensorMap tmSin,
                     const __grid_constant__ ScanParams p) {
  using Lay = WinLayout<kRope, kL3>;
  constexpr int S = Lay::stages;
  extern __shared__ __align__(1024) uint8_t win_smem[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ float4 s_agg[2][kWinWarps][2][32];  // per warp: zero-state aggregate of its 4 tokens
  __shared__ float4 s_carry[2][2][32];           // state after the previous sub-chunk
  __shared__ float4 s_wa[kWinWarps][2][32];      // warm-up sums A_w

  const int warp = warp_id();
  const int lane = lane_id();
  // CTA -> (segment, batch row, slice); neighbouring CTAs share a token range.
  // The CTAs of K slices (RoPE) come first, with their own segment length.
  const bool kgrp = static_cast<int>(blockIdx.x) < p.n_ctas_k;
  const int nds_g = kgrp ? p.nds_k : p.nds - p.nds_k;
  const int bid = kgrp ? static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x) - p.n_ctas_k;
  const int nss = p.B * nds_g;
  const int seg = bid / nss;
  const int ss = bid % nss;
  const int b = ss / nds_g;
  const int ds = (kgrp ? 0 : p.nds_k) + ss % nds_g;
  const int T = p.T;
  const int seg_len = kgrp ? p.seg_len_k : p.seg_len_v;
  const int s0 = seg * seg_len;
  const int s1 = min(s0 + seg_len, T);
  const int ws = max(0, s0 - p.win_tokens);
  const int nwarm = (s0 - ws) / kWinTok;                             // warm-up sub-chunks
  constexpr int kWT = Lay::warm_tiles;
  const int nwst = (nwarm + kWT - 1) / kWT;                          // warm-up stages
  const int nsub = nwst + (s1 - s0 + kWinTok - 1) / kWinTok;          // stage uses
  const int nk = p.D >> 1;
  const bool cta_has_k = ds * kSlice < nk;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 2);  // the producer's expect_tx arrival and its arrival after the gates
      mbar_init(&empty_bar[i], kWinWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kWinWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmY);
      if (kL3) tma_prefetch_desc(&tmY3);
      if (kRope && cta_has_k) {
        tma_prefetch_desc(&tmCos);
        tma_prefetch_desc(&tmSin);
      }
    }
    const uint32_t main_tx =
        kWinYBytes + (kL3 ? kWinYBytes : 0) + ((kRope && cta_has_k) ? 2 * kWinRopeBytes : 0);
    const int b3 = p.l3_bcast ? 0 : b;
    const int rb = p.rope_bcast ? 0 : b;
    bool dead = false;
    // router logits of token (segment sub-chunk m) * kWinTok + 32 h + lane, loaded S stage uses ahead
    const float b20 = p.b2 ? p.b2[0] : 0.f, b21 = p.b2 ? p.b2[1] : 0.f, b22 = (kL3 && p.b2) ? p.b2[2] : 0.f;
    auto load_logits = [&](int m, int h, float (&lg)[3]) {
      const int t = s0 + m * kWinTok + 32 * h + lane;
      lg[0] = lg[1] = 0.f;
      lg[2] = -INFINITY;
      if (m >= 0 && t < s1) {
        const float* src = p.logits + ((int64_t)b * T + t) * p.L;
        lg[0] = __ldg(src);
        lg[1] = __ldg(src + 1);
        if (kL3) lg[2] = __ldg(src + 2);
      }
    };
    float lgq[S][kWinHalves][3];
#pragma unroll
    for (int a = 0; a < S; ++a) {
#pragma unroll
      for (int h = 0; h < kWinHalves; ++h) load_logits(a - nwst, h, lgq[a][h]);
    }
    int st = 0;
    uint32_t phase = 0;  // parity of this use of stage st; the previous use had phase ^ 1
    for (int k = 0; k < nsub; ++k) {
      if (k >= S && !dead) dead = !mbar_wait(&empty_bar[st], phase ^ 1u, p.status);
      uint8_t* stage = win_smem + st * Lay::stage;
      const bool in_seg = k >= nwst;
      if (lane == 0 && !in_seg) {
        const int tile0 = k * kWT;
        const int ntile = min(kWT, nwarm - tile0);
        mbar_arrive_expect_tx(&full_bar[st], static_cast<uint32_t>(ntile * kWinYBytes));
        for (int i = 0; i < ntile; ++i)
          tma_load_3d(stage + i * kWinYBytes, &tmY, &full_bar[st], ds * kSlice, ws + (tile0 + i) * kWinTok, b);
      }
      const int t0 = s0 + (k - nwst) * kWinTok;
      if (lane == 0 && in_seg) {
        mbar_arrive_expect_tx(&full_bar[st], main_tx);
        tma_load_3d(stage + Lay::y, &tmY, &full_bar[st], ds * kSlice, t0, b);
        if (kL3) tma_load_3d(stage + Lay::y3, &tmY3, &full_bar[st], ds * kSlice, min(t0, p.T3 - 1), b3);
        if (kRope && cta_has_k) {
          tma_load_3d(stage + Lay::cs, &tmCos, &full_bar[st], 0, t0, rb);
          tma_load_3d(stage + Lay::sn, &tmSin, &full_bar[st], 0, t0, rb);
        }
      }
      if (in_seg) {
#pragma unroll
        for (int h = 0; h < kWinHalves; ++h) {
          // gate of token t0 + 32 h + lane: lam0, lam1 (1 - beta), lam2
          const int t = t0 + 32 * h + lane;
          float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
          if (t < s1) {
            float a0 = lgq[0][h][0] + b20, a1 = lgq[0][h][1] + b21, a2 = kL3 ? lgq[0][h][2] + b22 : -INFINITY;
            const float mx = fmaxf(fmaxf(a0, a1), a2);
            a0 = __expf(a0 - mx);
            a1 = __expf(a1 - mx);
            a2 = kL3 ? __expf(a2 - mx) : 0.f;
            const float inv = 1.f / (a0 + a1 + a2);
            a0 *= inv;
            a1 *= inv;
            a2 *= inv;
            if (p.lam != nullptr && ds == 0) {
              float* dstl = p.lam + ((int64_t)b * T + t) * p.L;
              dstl[0] = a0;
              dstl[1] = a1;
              if (kL3) dstl[2] = a2;
            }
            g = make_float4(a0, a1 * p.one_minus_beta, a2, 0.f);
          }
          reinterpret_cast<float4*>(stage + Lay::gate)[32 * h + lane] = g;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_bar[st]);
      // shift the logits queue by one stage use
#pragma unroll
      for (int a = 0; a + 1 < S; ++a) {
#pragma unroll
        for (int h = 0; h < kWinHalves; ++h) {
#pragma unroll
          for (int i = 0; i < 3; ++i) lgq[a][h][i] = lgq[a + 1][h][i];
        }
      }
#pragma unroll
      for (int h = 0; h < kWinHalves; ++h) load_logits(k + S - nwst, h, lgq[S - 1][h]);
      if (++st == S) {
        st = 0;
        phase ^= 1u;
      }
    }
    // no load may still be in flight when the CTA exits
    for (int k = max(0, nsub - S); k < nsub; ++k)
      if (!dead) dead = !mbar_wait(&full_bar[k % S], static_cast<uint32_t>(k / S) & 1u, p.status);
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int hh = lane >> 4;
  const int q = lane & 15;
  const int col = hh * 128 + 4 * q;  // this lane's first channel in the slice (the second block is col + 64)
  const int ch = ds * kSlice + col;
  const bool is_k = ch < nk;
  const int head = (is_k ? ch : ch - nk) >> 7;
  __nv_bfloat16* out = (is_k ? p.kv_k : p.kv_v) + (int64_t)b * p.kv_sb + (int64_t)head * p.kv_sh +
                       (int64_t)p.t_offset * p.kv_st + 4 * q;
  float bias[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (kBias) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + ch));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + ch + 64));
    bias[0] = b0.x; bias[1] = b0.y; bias[2] = b0.z; bias[3] = b0.w;
    bias[4] = b1.x; bias[5] = b1.y; bias[6] = b1.z; bias[7] = b1.w;
  }
  const float beta = p.beta;
  const float b4 = p.beta4;
  float pw[kWinTpw];  // beta^(j + 1)
  pw[0] = beta;
#pragma unroll
  for (int j = 1; j < kWinTpw; ++j) pw[j] = pw[j - 1] * beta;
  const int r0 = warp * kWinTpw;  // this warp's first row of a sub-chunk
  bool dead = false;

  // warm-up: this warp's running sum of its aggregates
  float A[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int st = 0;          // stage of sub-chunk k
  uint32_t phase = 0;  // parity of its use of that stage
  auto next_stage = [&]() {
    if (++st == S) {
      st = 0;
      phase ^= 1u;
    }
  };
  int k = 0;
  for (; k < nwst; ++k, next_stage()) {
    if (!dead) dead = !mbar_wait(&full_bar[st], phase, p.status);
    const int ntile = min(kWT, nwarm - k * kWT);
    const uint8_t* yb = win_smem + st * Lay::stage + r0 * kWinRowBytes + col * 2;
    uint2 lo[kWT][kWinTpw], hi[kWT][kWinTpw];
#pragma unroll
    for (int i = 0; i < kWT; ++i) {
      if (i < ntile) {
#pragma unroll
        for (int j = 0; j < kWinTpw; ++j) {
          lo[i][j] = *reinterpret_cast<const uint2*>(yb + i * kWinYBytes + j * kWinRowBytes);
          hi[i][j] = *reinterpret_cast<const uint2*>(yb + i * kWinYBytes + j * kWinRowBytes + 128);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
#pragma unroll
    for (int i = 0; i < kWT; ++i) {
      if (i < ntile) {
        float a[8];
#pragma unroll
        for (int j = 0; j < kWinTpw; ++j) {
          float yf[8];
          unpack_lohi(lo[i][j], hi[i][j], yf);
#pragma unroll
          for (int c = 0; c < 8; ++c) a[c] = j == 0 ? yf[c] : fmaf(beta, a[c], yf[c]);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) A[c] = fmaf(p.beta32, A[c], a[c]);
      }
    }
  }
  put8(s_wa[warp], lane, A);  // read after the first barrier of the segment

  // RoPE in this CTA: 0 none (V slice), 1 every lane (K slice), 2 the lanes of K heads
  const int rope_mode = !kRope ? 0 : (!cta_has_k ? 0 : (ds * kSlice + kSlice <= nk ? 1 : 2));

  // the segment
  for (int km = 0; k < nsub; ++k, ++km, next_stage()) {
    if (!dead) dead = !mbar_wait(&full_bar[st], phase, p.status);
    const uint8_t* sb = win_smem + st * Lay::stage;
    const int t0 = s0 + km * kWinTok;
    constexpr bool kKeepY = kWinTpw <= 4;  // 8 tokens a warp read y again in the blend (registers)
    float yf[kKeepY ? kWinTpw : 1][8];
    float u[kWinTpw][8];
#pragma unroll
    for (int j = 0; j < kWinTpw; ++j) {
      const uint8_t* row = sb + Lay::y + (r0 + j) * kWinRowBytes + col * 2;
      float f[8];
      unpack_lohi(*reinterpret_cast<const uint2*>(row), *reinterpret_cast<const uint2*>(row + 128), f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        u[j][c] = j == 0 ? f[c] : fmaf(beta, u[j - 1][c], f[c]);
        if constexpr (kKeepY) yf[j][c] = f[c];
      }
    }
    const int par = km & 1;
    put8(s_agg[par][warp], lane, u[kWinTpw - 1]);
    named_bar_sync(1, kWinWarps * 32);

    // state entering this warp's first token
    float s[8];
    if (km == 0) {
#pragma unroll
      for (int c = 0; c < 8; ++c) s[c] = 0.f;
#pragma unroll
      for (int v = 0; v < kWinWarps; ++v) {
        float a[8];
        get8(s_wa[v], lane, a);
#pragma unroll
        for (int c = 0; c < 8; ++c) s[c] = fmaf(b4, s[c], a[c]);
      }
    } else {
      get8(s_carry[par], lane, s);
    }
    for (int v = 0; v < warp; ++v) {
      float a[8];
      get8(s_agg[par][v], lane, a);
#pragma unroll
      for (int c = 0; c < 8; ++c) s[c] = fmaf(b4, s[c], a[c]);
    }
    if (warp == kWinWarps - 1) {
      float cnext[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) cnext[c] = fmaf(b4, s[c], u[kWinTpw - 1][c]);
      put8(s_carry[par ^ 1], lane, cnext);
    }

    // blend, bias, RoPE, head-split store (RoPE mode fixed per CTA at compile time)
    __nv_bfloat16* dst0 = out + (int64_t)(t0 + r0) * p.kv_st;
    auto blend = [&](auto rope_c) {
      constexpr int rm = decltype(rope_c)::value;
#pragma unroll
    for (int j = 0; j < kWinTpw; ++j) {
      const int t = t0 + r0 + j;
      const float4 g = reinterpret_cast<const float4*>(sb + Lay::gate)[r0 + j];
      float yv[8];
      if constexpr (kKeepY) {
#pragma unroll
        for (int c = 0; c < 8; ++c) yv[c] = yf[j][c];
      } else {
        const uint8_t* row = sb + Lay::y + (r0 + j) * kWinRowBytes + col * 2;
        unpack_lohi(*reinterpret_cast<const uint2*>(row), *reinterpret_cast<const uint2*>(row + 128), yv);
      }
      float o[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float uc = fmaf(pw[j], s[c], u[j][c]);
        o[c] = fmaf(g.y, uc, fmaf(g.x, yv[c], bias[c]));
      }
      if (kL3) {
        const int r3 = min(t, p.T3 - 1) - min(t0, p.T3 - 1);
        const uint8_t* row3 = sb + Lay::y3 + r3 * kWinRowBytes + col * 2;
        float y3f[8];
        unpack_lohi(*reinterpret_cast<const uint2*>(row3), *reinterpret_cast<const uint2*>(row3 + 128), y3f);
#pragma unroll
        for (int c = 0; c < 8; ++c) o[c] = fmaf(g.z, y3f[c], o[c]);
      }
      if (kRope && (rm == 1 || (rm == 2 && is_k))) {
        const float* cr = reinterpret_cast<const float*>(sb + Lay::cs) + (r0 + j) * 128 + 4 * q;
        const float* sr = reinterpret_cast<const float*>(sb + Lay::sn) + (r0 + j) * 128 + 4 * q;
        const float4 cl = *reinterpret_cast<const float4*>(cr);
        const float4 chv = *reinterpret_cast<const float4*>(cr + 64);
        const float4 sl = *reinterpret_cast<const float4*>(sr);
        const float4 shv = *reinterpret_cast<const float4*>(sr + 64);
        const float cla[4] = {cl.x, cl.y, cl.z, cl.w}, cha[4] = {chv.x, chv.y, chv.z, chv.w};
        const float sla[4] = {sl.x, sl.y, sl.z, sl.w}, sha[4] = {shv.x, shv.y, shv.z, shv.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float lo = o[c], hi = o[c + 4];
          o[c] = fmaf(-hi, sla[c], lo * cla[c]);      // x1 cos - x2 sin
          o[c + 4] = fmaf(lo, sha[c], hi * cha[c]);   // x2 cos + x1 sin
        }
      }
      if (t < s1) {
        __nv_bfloat16* dst = dst0 + (int64_t)j * p.kv_st;
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
        *reinterpret_cast<uint2*>(dst + 64) = make_uint2(pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
      }
    }
    };
    if (rope_mode == 1)
      blend(std::integral_constant<int, 1>{});
    else if (rope_mode == 0)
      blend(std::integral_constant<int, 0>{});
    else
      blend(std::integral_constant<int, 2>{});
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
  }
}

// The layer's stage 1 for short inputs (T <= kSmallT tokens, no carried
// state), e.g. a decode step: one warp per (batch row, 256-channel slice) scans
// the tokens one after another. Lanes hold channels as in kv_window_kernel (d
// and d + 64 of one head), the state is in u units, and each lane computes the
// gate of the current token itself (a broadcast read of the logits); nothing
// is staged, so the whole stage is one short wave of warps.
constexpr int kSmallT = 32;

template <bool kRope, bool kBias, bool kL3>
__global__ void __launch_bounds__(32) kv_small_kernel(const __grid_constant__ ScanParams p) {
  const int lane = lane_id();
  const int b = static_cast<int>(blockIdx.x) / p.nds;
  const int ds = static_cast<int>(blockIdx.x) % p.nds;
  const int hh = lane >> 4;
  const int q = lane & 15;
  const int col = hh * 128 + 4 * q;
  const int ch = ds * kSlice + col;
  const int nk = p.D >> 1;
  const bool is_k = ch < nk;
  const int head = (is_k ? ch : ch - nk) >> 7;
  __nv_bfloat16* out = (is_k ? p.kv_k : p.kv_v) + (int64_t)b * p.kv_sb + (int64_t)head * p.kv_sh +
                       (int64_t)p.t_offset * p.kv_st + 4 * q;
  float bias[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (kBias) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + ch));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.kv_bias + ch + 64));
    bias[0] = b0.x; bias[1] = b0.y; bias[2] = b0.z; bias[3] = b0.w;
    bias[4] = b1.x; bias[5] = b1.y; bias[6] = b1.z; bias[7] = b1.w;
  }
  const float b20 = p.b2 ? p.b2[0] : 0.f, b21 = p.b2 ? p.b2[1] : 0.f, b22 = (kL3 && p.b2) ? p.b2[2] : 0.f;
  const __nv_bfloat16* yb = p.x + (int64_t)b * p.x_sb + ch;
  float u[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < p.T; ++t) {
    float yf[8];
    const __nv_bfloat16* yr = yb + (int64_t)t * p.x_st;
    unpack_lohi(__ldg(reinterpret_cast<const uint2*>(yr)), __ldg(reinterpret_cast<const uint2*>(yr + 64)), yf);
    // gate of token t (every lane, the same values)
    const int64_t row = (int64_t)b * p.T + t;
    const float* lg = p.logits + row * p.L;
    float a0 = __ldg(lg) + b20, a1 = __ldg(lg + 1) + b21, a2 = kL3 ? __ldg(lg + 2) + b22 : -INFINITY;
    const float mx = fmaxf(fmaxf(a0, a1), a2);
    a0 = __expf(a0 - mx);
    a1 = __expf(a1 - mx);
    a2 = kL3 ? __expf(a2 - mx) : 0.f;
    const float inv = 1.f / (a0 + a1 + a2);
    a0 *= inv;
    a1 *= inv;
    a2 *= inv;
    if (p.lam != nullptr && ds == 0 && lane == 0) {
      p.lam[row * p.L] = a0;
      p.lam[row * p.L + 1] = a1;
      if (kL3) p.lam[row * p.L + 2] = a2;
    }
    const float g1 = a1 * p.one_minus_beta;
    float o[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      u[c] = fmaf(p.beta, u[c], yf[c]);
      o[c] = fmaf(g1, u[c], fmaf(a0, yf[c], bias[c]));
    }
    if (kL3) {
      const int t3 = t < p.T3 ? t : p.T3 - 1;
      const __nv_bfloat16* r3 = p.l3 + (int64_t)b * p.l3_sb + (int64_t)t3 * p.l3_st + ch;
      float y3f[8];
      unpack_lohi(__ldg(reinterpret_cast<const uint2*>(r3)), __ldg(reinterpret_cast<const uint2*>(r3 + 64)), y3f);
#pragma unroll
      for (int c = 0; c < 8; ++c) o[c] = fmaf(a2, y3f[c], o[c]);
    }
    if (kRope && is_k) {
      const float* cr = p.rope_cos + (int64_t)(p.rope_bcast ? 0 : b) * p.rope_sb + (int64_t)t * p.rope_st + 4 * q;
      const float* sr = p.rope_sin + (int64_t)(p.rope_bcast ? 0 : b) * p.rope_sb + (int64_t)t * p.rope_st + 4 * q;
      const float4 cl = __ldg(reinterpret_cast<const float4*>(cr));
      const float4 chv = __ldg(reinterpret_cast<const float4*>(cr + 64));
      const float4 sl = __ldg(reinterpret_cast<const float4*>(sr));
      const float4 shv = __ldg(reinterpret_cast<const float4*>(sr + 64));
      const float cla[4] = {cl.x, cl.y, cl.z, cl.w}, cha[4] = {chv.x, chv.y, chv.z, chv.w};
      const float sla[4] = {sl.x, sl.y, sl.z, sl.w}, sha[4] = {shv.x, shv.y, shv.z, shv.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float lo = o[c], hi = o[c + 4];
        o[c] = fmaf(-hi, sla[c], lo * cla[c]);      // x1 cos - x2 sin
        o[c + 4] = fmaf(lo, sha[c], hi * cha[c]);   // x2 cos + x1 sin
      }
    }
    __nv_bfloat16* dst = out + (int64_t)t * p.kv_st;
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
    *reinterpret_cast<uint2*>(dst + 64) = make_uint2(pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

template <bool kRope, bool kBias, bool kL3>
int launch_kv_small_t(const ScanParams& p, cudaStream_t stream) {
  kv_small_kernel<kRope, kBias, kL3><<<(unsigned)(p.B * p.nds), 32, 0, stream>>>(p);
  return check_cuda(cudaGetLastError(), "kv_small launch");
}

template <bool kRope, bool kBias, bool kL3>
int launch_kv_window_t(const CUtensorMap& tmY, const CUtensorMap& tmY3, const CUtensorMap& tmCos,
                       const CUtensorMap& tmSin, const ScanParams& p, int grid, cudaStream_t stream) {
  constexpr int smem = WinLayout<kRope, kL3>::bytes;
  auto kern = kv_window_kernel<kRope, kBias, kL3>;
  int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                      "kv_window attr");
  if (rc) return rc;
  kern<<<grid, kWinThreads, smem, stream>>>(tmY, tmY3, tmCos, tmSin, p);
  return check_cuda(cudaGetLastError(), "kv_window launch");
}

}  // namespace

// FMKA_SCAN_GENERAL=1 sends the layer's K/V scan to the general kernel too
// (for comparisons; both compute the same function).
static bool scan_general_forced() {
  static const bool on = [] {
    const char* e = std::getenv("FMKA_SCAN_GENERAL");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}

// FMKA_SCAN_WINDOW=0 keeps the layer's K/V scan on kv_scan_kernel (the
// chunk-parallel look-back form) instead of kv_window_kernel / kv_small_kernel.
static bool scan_window_off() {
  static const bool off = [] {
    const char* e = std::getenv("FMKA_SCAN_WINDOW");
    return e != nullptr && e[0] == '0';
  }();
  return off;
}

// Cost of a V-slice token relative to a K-slice token (RoPE) in kv_window_kernel,
// used to split the grid between the two; FMKA_WIN_V_COST overrides it.
static double win_v_cost() {
  static const double c = [] {
    const char* e = std::getenv("FMKA_WIN_V_COST");
    const double v = e ? std::atof(e) : 0.0;
    return v > 0.05 && v <= 4.0 ? v : 0.8;  // measured at batch 2 and 4 x 8192 (0.8-1.0; 0.5-1.05 before)
  }();
  return c;
}

// Window of kv_window_kernel: the fewest whole sub-chunks W (at most 64) with
// |beta|^W < 2^-40; 0 when the memory is longer than that.
static int window_tokens(float beta) {
  const double bc = std::fabs(__builtin_powi((double)beta, kWinTok));
  double w = 1.0;
  for (int k = 1; k <= 64; ++k) {
    w *= bc;
    if (w < 0x1p-40) return k * kWinTok;
  }
  return 0;
}

// The layer's K/V scan through kv_window_kernel; returns -1 (nothing launched)
// when a tensor does not suit TMA, so that the caller takes another kernel.
// The layer's K/V scan for short inputs through kv_small_kernel; returns -1
// (nothing launched) when it does not apply.
static int launch_kv_small(ScanParams p, cudaStream_t stream) {
  if (p.T > kSmallT || p.D % kSlice != 0 || scan_window_off()) return -1;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const bool rope = p.rope_cos != nullptr, bias = p.kv_bias != nullptr, l3v = p.l3 != nullptr;
  if (rope && ((p.rope_st % 4) || (p.rope_sb % 4) || !al16(p.rope_cos) || !al16(p.rope_sin))) return -1;
  if (bias && !al16(p.kv_bias)) return -1;
  if ((int64_t)p.B * p.nds > 0x7FFFFFFF) return -1;
  p.rope_bcast = (p.rope_sb == 0 || p.B == 1) ? 1 : 0;
  if (rope)
    return bias ? (l3v ? launch_kv_small_t<true, true, true>(p, stream) : launch_kv_small_t<true, true, false>(p, stream))
                : (l3v ? launch_kv_small_t<true, false, true>(p, stream) : launch_kv_small_t<true, false, false>(p, stream));
  return bias ? (l3v ? launch_kv_small_t<false, true, true>(p, stream) : launch_kv_small_t<false, true, false>(p, stream))
              : (l3v ? launch_kv_small_t<false, false, true>(p, stream) : launch_kv_small_t<false, false, false>(p, stream));
}

static int launch_kv_window(ScanParams p, cudaStream_t stream) {
  const int W = window_tokens(p.beta);
  if (W == 0 || p.D % kSlice != 0 || scan_window_off()) return -1;
  const bool rope = p.rope_cos != nullptr, bias = p.kv_bias != nullptr, l3v = p.l3 != nullptr;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (rope && ((p.rope_st % 4) || (p.rope_sb % 4) || !al16(p.rope_cos) || !al16(p.rope_sin))) return -1;
  if (bias && !al16(p.kv_bias)) return -1;
  if (p.x_st < p.D || (l3v && p.l3_st < p.D)) return -1;
  CUtensorMap tmY, tmY3, tmCos, tmSin;
  {
    const uint64_t dims[3] = {(uint64_t)p.D, (uint64_t)p.T, (uint64_t)p.B};
    const uint64_t strides[2] = {(uint64_t)p.x_st * 2, (uint64_t)(p.B > 1 ? p.x_sb : (int64_t)p.T * p.x_st) * 2};
    const uint32_t box[3] = {(uint32_t)kSlice, (uint32_t)kWinTok, 1u};
    if (make_tmap_bf16(&tmY, p.x, 3, dims, strides, box, false) != kOk) return -1;
  }
  tmY3 = tmY;
  p.l3_bcast = 0;
  if (l3v) {
    p.l3_bcast = (p.l3_sb == 0 || p.B == 1) ? 1 : 0;
    const uint64_t dims[3] = {(uint64_t)p.D, (uint64_t)p.T3, (uint64_t)(p.l3_bcast ? 1 : p.B)};
    const uint64_t strides[2] = {(uint64_t)p.l3_st * 2,
                                 (uint64_t)(p.l3_bcast ? (int64_t)p.T3 * p.l3_st : p.l3_sb) * 2};
    const uint32_t box[3] = {(uint32_t)kSlice, (uint32_t)kWinTok, 1u};
    if (make_tmap_bf16(&tmY3, p.l3, 3, dims, strides, box, false) != kOk) return -1;
  }
  tmCos = tmSin = tmY;
  p.rope_bcast = 0;
  if (rope) {
    p.rope_bcast = (p.rope_sb == 0 || p.B == 1) ? 1 : 0;
    const uint64_t dims[3] = {128u, (uint64_t)p.T, (uint64_t)(p.rope_bcast ? 1 : p.B)};
    const uint64_t strides[2] = {(uint64_t)p.rope_st * 4,
                                 (uint64_t)(p.rope_bcast ? (int64_t)p.T * p.rope_st : p.rope_sb) * 4};
    const uint32_t box[3] = {128u, (uint32_t)kWinTok, 1u};
    if (make_tmap_f32(&tmCos, p.rope_cos, 3, dims, strides, box) != kOk) return -1;
    if (make_tmap_f32(&tmSin, p.rope_sin, 3, dims, strides, box) != kOk) return -1;
  }
  // Segments: one CTA per SM over all (batch row, slice, segment) triples.
  // Slices with K heads (RoPE) cost more per token than V-only slices, so the
  // two groups get their own segment lengths, split to even out CTA times:
  // a V token costs about kv_cost of a K token.
  const int sms = num_sms_current_device();
  const int nds_k = (p.D / 2 + kSlice - 1) / kSlice;
  const int nds_v = p.nds - nds_k;
  const double kv_cost = rope ? win_v_cost() : 1.0;
  auto seg_for = [&](int nseg) {
    int len = (p.T + nseg - 1) / nseg;
    return (len + kWinTok - 1) / kWinTok * kWinTok;
  };
  int best_k = 1, best_v = 1;
  double best = 1e300;
  for (int nk_seg = 1; nk_seg <= sms; ++nk_seg) {
    const int64_t used = (int64_t)p.B * nds_k * nk_seg;
    if (used > sms && nk_seg > 1) break;
    int nv_seg = 1;
    if (nds_v > 0) {
      const int64_t left = sms - used;
      if (left < (int64_t)p.B * nds_v && nk_seg > 1) break;  // the V slices would not fit in one wave
      nv_seg = left / ((int64_t)p.B * nds_v) > 1 ? (int)(left / ((int64_t)p.B * nds_v)) : 1;
    }
    const double tk = seg_for(nk_seg) + W;
    const double tv = nds_v > 0 ? (seg_for(nv_seg) + W) * kv_cost : 0.0;
    const double tmax = tk > tv ? tk : tv;
    if (tmax < best - 1e-9) {
      best = tmax;
      best_k = nk_seg;
      best_v = nv_seg;
    }
  }
  p.seg_len_k = seg_for(best_k);
  p.seg_len_v = seg_for(best_v);
  const int nseg_k = (p.T + p.seg_len_k - 1) / p.seg_len_k;
  const int nseg_v = (p.T + p.seg_len_v - 1) / p.seg_len_v;
  p.nds_k = nds_k;
  p.n_ctas_k = p.B * nds_k * nseg_k;
  const int64_t grid = (int64_t)p.n_ctas_k + (int64_t)p.B * nds_v * nseg_v;
  if (grid > 0x7FFFFFFF) return -1;
  p.win_tokens = W;
  p.beta4 = (float)__builtin_powi((double)p.beta, kWinTpw);
  p.beta32 = (float)__builtin_powi((double)p.beta, kWinTok);
  const int g = (int)grid;
  if (rope)
    return bias ? (l3v ? launch_kv_window_t<true, true, true>(tmY, tmY3, tmCos, tmSin, p, g, stream)
                       : launch_kv_window_t<true, true, false>(tmY, tmY3, tmCos, tmSin, p, g, stream))
                : (l3v ? launch_kv_window_t<true, false, true>(tmY, tmY3, tmCos, tmSin, p, g, stream)
                       : launch_kv_window_t<true, false, false>(tmY, tmY3, tmCos, tmSin, p, g, stream));
  return bias ? (l3v ? launch_kv_window_t<false, true, true>(tmY, tmY3, tmCos, tmSin, p, g, stream)
                     : launch_kv_window_t<false, true, false>(tmY, tmY3, tmCos, tmSin, p, g, stream))
              : (l3v ? launch_kv_window_t<false, false, true>(tmY, tmY3, tmCos, tmSin, p, g, stream)
                     : launch_kv_window_t<false, false, false>(tmY, tmY3, tmCos, tmSin, p, g, stream));
}

size_t route_ema_blend_workspace_bytes(int B, int T, int D) {
  const int64_t nds = (D + kSlice - 1) / kSlice;
  const int64_t nchunks = (T + kChunkT - 1) / kChunkT;
  const int64_t nrec = (int64_t)B * nds * nchunks;
  const int64_t flag_bytes = ((nrec * 4 + 256 + 255) / 256) * 256;  // ticket + flags, 256-aligned
  return (size_t)(flag_bytes + 2 * nrec * kSlice * 4);
}

size_t route_ema_blend_flag_bytes(int B, int T, int D) {
  const int64_t nds = (D + kSlice - 1) / kSlice;
  const int64_t nchunks = (T + kChunkT - 1) / kChunkT;
  const int64_t nrec = (int64_t)B * nds * nchunks;
  return (size_t)(((nrec * 4 + 256 + 255) / 256) * 256);
}

// K/V output of the blend (see ScanParams); null kv_k keeps the H output.
struct KvOut {
  __nv_bfloat16* k = nullptr;
  __nv_bfloat16* v = nullptr;
  int64_t sb = 0, sh = 0, st = 0;
  int t_offset = 0;
  const float* bias = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int64_t rope_sb = 0, rope_st = 0;
};

int launch_route_ema_blend(const __nv_bfloat16* x, int64_t x_sb, int64_t x_st, const __nv_bfloat16* l2,
                           int64_t l2_sb, int64_t l2_st, const float* logits,
                           const float* b2, const float* gate, int L, const __nv_bfloat16* l3, int64_t l3_sb,
                           int64_t l3_st, int T3, float beta, int B, int T, int D, __nv_bfloat16* h,
                           int64_t h_sb, int64_t h_st, float* lam, void* workspace, size_t workspace_bytes,
                           bool clear_flags, cudaStream_t stream, const float* ema_init, float* ema_final,
                           const KvOut* kv = nullptr) {
  if (B <= 0 || T <= 0 || D <= 0) return set_error(kErrInvalidArgument, "route_ema_blend: empty shape");
  if (l2 != nullptr && (ema_init != nullptr || ema_final != nullptr))
    return set_error(kErrInvalidArgument, "route_ema_blend: an EMA state needs the scan (no given L2)");
  if ((reinterpret_cast<uintptr_t>(ema_init) | reinterpret_cast<uintptr_t>(ema_final)) & 15u)
    return set_error(kErrInvalidArgument, "route_ema_blend: EMA states must be 16-byte aligned");
  if (D % 8 != 0) return set_error(kErrUnsupported, "route_ema_blend: d_model must be a multiple of 8");
  if (L < 2 || L > 3) return set_error(kErrInvalidArgument, "route_ema_blend: levels must be 2 or 3");
  if (L == 3 && (l3 == nullptr || T3 < 1))
    return set_error(kErrInvalidArgument, "route_ema_blend: 3 levels need an L3 memory with >= 1 row");
  if ((logits == nullptr) == (gate == nullptr))
    return set_error(kErrInvalidArgument, "route_ema_blend: pass exactly one of logits or gate");
  if ((x_st % 8) || (x_sb % 8) || (h_st % 8) || (h_sb % 8) || (l3 && ((l3_st % 8) || (l3_sb % 8))) ||
      (l2 && ((l2_st % 8) || (l2_sb % 8))))
    return set_error(kErrInvalidArgument, "route_ema_blend: strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(h) & 15u) ||
      (l3 && (reinterpret_cast<uintptr_t>(l3) & 15u)) || (l2 && (reinterpret_cast<uintptr_t>(l2) & 15u)))
    return set_error(kErrInvalidArgument, "route_ema_blend: tensors must be 16-byte aligned");
  const size_t need = route_ema_blend_workspace_bytes(B, T, D);
  if (l2 == nullptr && (workspace == nullptr || workspace_bytes < need))
    return set_error(kErrWorkspace, "route_ema_blend: workspace too small (need " + std::to_string(need) + " bytes)");
  if (l2 == nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return set_error(kErrInvalidArgument, "route_ema_blend: workspace must be 256-byte aligned");

  ScanParams p;
  p.x = x;
  p.x_sb = x_sb;
  p.x_st = x_st;
  p.l2 = l2;
  p.l2_sb = l2_sb;
  p.l2_st = l2_st;
  p.logits = logits;
  p.b2 = b2;
  p.gate = gate;
  p.L = L;
  p.l3 = (L == 3) ? l3 : nullptr;
  p.l3_sb = l3_sb;
  p.l3_st = l3_st;
  p.T3 = T3;
  p.beta = beta;
  p.one_minus_beta = 1.0f - beta;
  p.beta8 = (float)__builtin_powi((double)beta, 8);
  p.beta_chunk = (float)__builtin_powi((double)beta, kChunkT);
  // the shortest look-back whose first left-out weight beta^(kChunkT k) is
  // below 2^-40 (at most 32 chunks; otherwise the full look-back)
  p.lb_max = 0;
  {
    const double bc = std::fabs(__builtin_powi((double)beta, kChunkT));
    double w = 1.0;
    for (int k = 1; k <= 32; ++k) {
      w *= bc;
      if (w < 0x1p-40) {
        p.lb_max = k;
        break;
      }
    }
  }
  p.B = B;
  p.T = T;
  p.D = D;
  p.h = h;
  p.h_sb = h_sb;
  p.h_st = h_st;
  p.lam = lam;
  p.ema_init = ema_init;
  p.ema_final = ema_final;
  p.kv_k = nullptr;
  p.kv_v = nullptr;
  p.kv_bias = nullptr;
  p.rope_cos = p.rope_sin = nullptr;
  p.kv_sb = p.kv_sh = p.kv_st = 0;
  p.t_offset = 0;
  p.rope_sb = p.rope_st = 0;
  if (kv != nullptr) {
    p.kv_k = kv->k;
    p.kv_v = kv->v;
    p.kv_sb = kv->sb;
    p.kv_sh = kv->sh;
    p.kv_st = kv->st;
    p.t_offset = kv->t_offset;
    p.kv_bias = kv->bias;
    p.rope_cos = kv->rope_cos;
    p.rope_sin = kv->rope_sin;
    p.rope_sb = kv->rope_sb;
    p.rope_st = kv->rope_st;
  }
  p.nds = (D + kSlice - 1) / kSlice;
  p.nchunks = (T + kChunkT - 1) / kChunkT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t flag_bytes = route_ema_blend_flag_bytes(B, T, D);
  const int64_t nrec = (int64_t)B * p.nds * p.nchunks;
  p.ticket = reinterpret_cast<uint32_t*>(ws);
  p.flags = reinterpret_cast<uint32_t*>(ws + 256);
  p.agg = reinterpret_cast<float*>(ws + flag_bytes);
  p.inc = p.agg + nrec * kSlice;
  p.status = device_status_word();
  if (kv != nullptr && l2 == nullptr && ema_init == nullptr && ema_final == nullptr && logits != nullptr &&
      !scan_general_forced()) {
    // the layer's case: a short input (a decode step) scanned token by token in
    // one wave of warps, else the streaming kernel (no flags, no look-back)
    // when the tensors suit TMA
    int rc = launch_kv_small(p, stream);
    if (rc >= 0) return rc;
    rc = launch_kv_window(p, stream);
    if (rc >= 0) return rc;
  }
  if (clear_flags && l2 == nullptr) {
    int rc = check_cuda(cudaMemsetAsync(ws, 0, flag_bytes, stream), "route_ema_blend memset");
    if (rc) return rc;
  }
  const int64_t grid = nrec;
  if (grid > 0x7FFFFFFF) return set_error(kErrUnsupported, "route_ema_blend: problem too large");
  if (kv != nullptr && l2 == nullptr && p.lb_max > 0 && ema_init == nullptr && ema_final == nullptr &&
      logits != nullptr && D % kSlice == 0 && !scan_general_forced()) {
    // the layer's case: the specialised kernel
    const bool rope = p.rope_cos != nullptr, bias = p.kv_bias != nullptr, l3v = p.l3 != nullptr;
    auto kern = rope ? (bias ? (l3v ? kv_scan_kernel<true, true, true> : kv_scan_kernel<true, true, false>)
                             : (l3v ? kv_scan_kernel<true, false, true> : kv_scan_kernel<true, false, false>))
                     : (bias ? (l3v ? kv_scan_kernel<false, true, true> : kv_scan_kernel<false, true, false>)
                             : (l3v ? kv_scan_kernel<false, false, true> : kv_scan_kernel<false, false, false>));
    kern<<<(unsigned)grid, kThreads, 0, stream>>>(p);
    return check_cuda(cudaGetLastError(), "kv_scan launch");
  }
  route_ema_blend_kernel<<<(unsigned)grid, kThreads, 0, stream>>>(p);
  return check_cuda(cudaGetLastError(), "route_ema_blend launch");
}

// Stage 1 on the projected memory: Y = X [Wk ; Wv]^T (bf16 [B, T, 2*Hkv*128])
// in, K/V out. Because the EMA runs along tokens and the projection along
// channels, EMA(X) Wk^T = EMA(X Wk^T); and since the gate sums to one, the
// bias can be added after the blend: K = lam0 (X Wk^T) + lam1 EMA(X Wk^T) + bk
// equals (lam0 X + lam1 EMA(X)) Wk^T + bk, the reference's k_proj of the fused
// memory (mka/hf/attention.py:105-111). With a third level, y3 = L3 [Wk ; Wv]^T
// ([B, T3, 2*Hkv*128], row t uses min(t, T3 - 1)) adds lam2 * y3.
int launch_route_ema_blend_kv(const __nv_bfloat16* y, int64_t y_sb, int64_t y_st, const float* logits, const float* b2,
                              const __nv_bfloat16* y3, int64_t y3_sb, int64_t y3_st, int T3,
                              float beta, int B, int T, int Hkv, const float* bias, __nv_bfloat16* k_out,
                              __nv_bfloat16* v_out, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, int t_offset,
                              const float* rope_cos, const float* rope_sin, int64_t rope_sb, int64_t rope_st,
                              float* lam, const float* ema_init, float* ema_final, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream) {
  if (Hkv <= 0) return set_error(kErrInvalidArgument, "route_ema_blend_kv: no kv heads");
  if (k_out == nullptr || v_out == nullptr || logits == nullptr)
    return set_error(kErrInvalidArgument, "route_ema_blend_kv: null pointer");
  if ((kv_st % 8) || (kv_sh % 8) || (kv_sb % 8) || t_offset < 0 ||
      ((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) & 15u))
    return set_error(kErrInvalidArgument, "route_ema_blend_kv: K/V need 16-byte aligned rows");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return set_error(kErrInvalidArgument, "route_ema_blend_kv: pass both RoPE tables or neither");
  if (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 15u))
    return set_error(kErrInvalidArgument, "route_ema_blend_kv: bias must be 16-byte aligned");
  KvOut kv;
  kv.k = k_out;
  kv.v = v_out;
  kv.sb = kv_sb;
  kv.sh = kv_sh;
  kv.st = kv_st;
  kv.t_offset = t_offset;
  kv.bias = bias;
  kv.rope_cos = rope_cos;
  kv.rope_sin = rope_sin;
  kv.rope_sb = rope_sb;
  kv.rope_st = rope_st;
  const int L = y3 != nullptr ? 3 : 2;
  return launch_route_ema_blend(y, y_sb, y_st, nullptr, 0, 0, logits, b2, nullptr, L, y3, y3_sb, y3_st, T3, beta, B,
                                T, 2 * Hkv * 128, nullptr, 0, 0, lam, workspace, workspace_bytes, true, stream,
                                ema_init, ema_final, &kv);
}

// ---------------------------------------------------------------------------
// Scratch without allocation.
//
// Some callers cannot allocate device memory when they call into this library:
// a serving runtime that reserved all of the GPU's memory for its own pools at
// start-up, a real-time path where cudaMalloc's implicit synchronisation is not
// acceptable, or a plain C program that links only this library and has no
// allocator of its own. For them the scan's scratch (chunk ticket, look-back
// flags and the per-chunk aggregate/inclusive states) lives in this fixed
// device array instead of a caller-provided workspace. Every GPU that loads the
// library holds the array until the process exits.
//
// In host code `g_route_scan_scratch` only names a host-side stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress, once per device,
// with that device current (the first call on a device does it, so make that
// first call before any stream capture). The address is kept for the life of
// the process; a cudaDeviceReset of that device invalidates it, so such a
// caller unloads and reloads the library. Every call shares the array and it
// keeps the previous call's contents: the flag region is cleared by a memset on
// the calling stream before each launch, and calls that overlap on the GPU (on
// different streams) race on the array.
// ---------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) uint8_t g_route_scan_scratch[kStaticScratchBytes];

namespace {
std::mutex g_static_scratch_mu;
void* g_static_scratch_dev[64] = {nullptr};
}  // namespace

size_t route_ema_blend_static_scratch_bytes() { return kStaticScratchBytes; }

int launch_route_ema_blend_static_scratch(const __nv_bfloat16* x, int64_t x_sb, int64_t x_st, const float* logits,
                                          const float* b2, const float* gate, int L, const __nv_bfloat16* l3,
                                          int64_t l3_sb, int64_t l3_st, int T3, float beta, int B, int T, int D,
                                          __nv_bfloat16* h, int64_t h_sb, int64_t h_st, float* lam,
                                          cudaStream_t stream) {
  if (B <= 0 || T <= 0 || D <= 0) return set_error(kErrInvalidArgument, "route_ema_blend_noalloc: empty shape");
  const size_t need = route_ema_blend_workspace_bytes(B, T, D);
  if (need > kStaticScratchBytes)
    return set_error(kErrUnsupported, "route_ema_blend_noalloc: this shape needs " + std::to_string(need) +
                                          " bytes of scratch, more than the " + std::to_string(kStaticScratchBytes) +
                                          "-byte static array; use fmka_route_ema_blend with a workspace");
  int dev = -1;
  int rc = check_cuda(cudaGetDevice(&dev), "route_ema_blend_noalloc: current device");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return set_error(kErrDevice, "route_ema_blend_noalloc: device index out of range");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_static_scratch_mu);
    if (g_static_scratch_dev[dev] == nullptr) {
      void* ptr = nullptr;
      rc = check_cuda(cudaGetSymbolAddress(&ptr, g_route_scan_scratch), "route_ema_blend_noalloc: scratch address");
      if (rc) return rc;
      g_static_scratch_dev[dev] = ptr;
    }
    scratch = g_static_scratch_dev[dev];
  }
  return launch_route_ema_blend(x, x_sb, x_st, nullptr, 0, 0, logits, b2, gate, L, l3, l3_sb, l3_st, T3, beta, B, T,
                                D, h, h_sb, h_st, lam, scratch, kStaticScratchBytes, /*clear_flags=*/true, stream,
                                nullptr, nullptr);
}

}  // namespace fmka
