// L3 chunk recall: the retrieval that produces the L3 memory R of the route
// blend from a bank of historical chunks.
//
// The reference describes this tier (mka/config/memory_hierarchy.py:1-10:
// "L3 - DRAM (vectorized hash, chunk recall): long-term retrieval /
// historical blocks"; l3_dram_chunk_recall and l3_recall_top_r, "top-R chunks
// per query", lines 30-34) and implements none of it: its layers take R from
// the caller (mka/layers/fastmka.py:84-89). The algorithm here is this
// package's own, built from that description:
//
//   1. the queries are block summaries: q_j = mean of x over query block j
//      (block_len tokens, the last block partial), rounded to bf16;
//   2. scores s_jc = q_j . key_c against every chunk key of the bank (a tcgen05
//      GEMM with an fp32 output, fmka_gemm_bf16_f32out);
//   3. the R best chunks of each block (ties: the lower chunk index first) and
//      weights softmax(scale * s) over those R;
//   4. R[b, t, :] = sum_r w_jr value_{c_jr} for every token t of block j.
//
// Kernels: block_mean_kernel (HBM-bound reduction), topr_kernel (one CTA per
// block row: each thread keeps a sorted top list of its strided columns in
// registers, the lists are merged by rounds of a shuffle argmax, per warp and
// then across the warps),
// recall_gather_kernel (each CTA forms one block's 256-channel slice of the
// weighted sum once and writes it to every token of the block).
#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

constexpr int kRecallSlice = 256;  // channels per CTA: 32 lanes x 8
constexpr int kRecallWarps = 8;
constexpr int kTopRUnroll = 4;  // float4 loads in flight per lane in topr_kernel

__device__ __forceinline__ void unpack8f(const uint4& u, float (&f)[8]) {
  f[0] = bf16lo_to_f32(u.x);
  f[1] = bf16hi_to_f32(u.x);
  f[2] = bf16lo_to_f32(u.y);
  f[3] = bf16hi_to_f32(u.y);
  f[4] = bf16lo_to_f32(u.z);
  f[5] = bf16hi_to_f32(u.z);
  f[6] = bf16lo_to_f32(u.w);
  f[7] = bf16hi_to_f32(u.w);
}

// q[b * nq + j, d] = bf16(mean over t in block j of x[b, t, d]).
__global__ void __launch_bounds__(kRecallWarps * 32) block_mean_kernel(const __nv_bfloat16* __restrict__ x,
                                                                       int64_t x_sb, int64_t x_st, int T, int D,
                                                                       int L, int nq, __nv_bfloat16* __restrict__ q,
                                                                       int64_t ldq) {
  __shared__ float4 part[kRecallWarps][2][32];
  const int row = blockIdx.x;  // b * nq + j
  const int b = row / nq;
  const int j = row % nq;
  const int warp = warp_id();
  const int lane = lane_id();
  const int d0 = blockIdx.y * kRecallSlice + lane * 8;
  const int t0 = j * L;
  const int t1 = min(t0 + L, T);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (d0 < D) {
    const __nv_bfloat16* xb = x + (int64_t)b * x_sb + d0;
    for (int t = t0 + warp; t < t1; t += kRecallWarps) {
      float f[8];
      unpack8f(__ldcs(reinterpret_cast<const uint4*>(xb + (int64_t)t * x_st)), f);
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] += f[c];
    }
  }
  part[warp][0][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  part[warp][1][lane] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  __syncthreads();
  if (warp == 0 && d0 < D) {
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kRecallWarps; ++w) {
      const float4 a = part[w][0][lane], c = part[w][1][lane];
      s[0] += a.x; s[1] += a.y; s[2] += a.z; s[3] += a.w;
      s[4] += c.x; s[5] += c.y; s[6] += c.z; s[7] += c.w;
    }
    const float inv = 1.f / (float)(t1 - t0);
    uint4 o;
    o.x = pack_bf16x2(s[0] * inv, s[1] * inv);
    o.y = pack_bf16x2(s[2] * inv, s[3] * inv);
    o.z = pack_bf16x2(s[4] * inv, s[5] * inv);
    o.w = pack_bf16x2(s[6] * inv, s[7] * inv);
    *reinterpret_cast<uint4*>(q + (int64_t)row * ldq + d0) = o;
  }
}

// (v, i) ranks before (w, k): larger score first, the lower index on ties.
__device__ __forceinline__ bool ranks_before(float v, int i, float w, int k) {
  return v > w || (v == w && i < k);
}

// One CTA per row of scores [M, N]: the R (<= kMax) best columns, sorted, and
// softmax(scale * score) over them. Each thread keeps a sorted list of the best
// kMax of its columns in registers (columns strided by the CTA, 16-byte loads,
// kTopRUnroll in flight); each warp merges its 32 lists by R rounds of a
// shuffle argmax into shared memory; warp 0 merges the 8 warp lists the same
// way and writes the result.
template <int kMax>
__global__ void __launch_bounds__(kRecallWarps * 32) topr_kernel(const float* __restrict__ scores, int64_t lds,
                                                                 int M, int N, int R, float scale,
                                                                 int* __restrict__ idx, float* __restrict__ w) {
  __shared__ float s_v[kRecallWarps][kMax];
  __shared__ int s_i[kRecallWarps][kMax];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = warp_id();
  const int lane = lane_id();
  constexpr int kThreads = kRecallWarps * 32;
  float v[kMax];
  int ix[kMax];
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    v[i] = -INFINITY;
    ix[i] = 0x7fffffff;
  }
  const float* sr = scores + (int64_t)row * lds;
  auto offer = [&](float cv, int ci) {
    if (!ranks_before(cv, ci, v[kMax - 1], ix[kMax - 1])) return;
    // insertion into the sorted list, branch-free
#pragma unroll
    for (int i = 0; i < kMax; ++i) {
      const bool bt = ranks_before(cv, ci, v[i], ix[i]);
      const float tv = bt ? cv : v[i];
      const int ti = bt ? ci : ix[i];
      cv = bt ? v[i] : cv;
      ci = bt ? ix[i] : ci;
      v[i] = tv;
      ix[i] = ti;
    }
  };
  int c_scalar = 0;
  if (((lds & 3) == 0) && ((reinterpret_cast<uintptr_t>(scores) & 15u) == 0)) {
    const int n4 = N >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(sr);
    for (int base = tid; base < n4; base += kThreads * kTopRUnroll) {
      float4 buf[kTopRUnroll];
#pragma unroll
      for (int u = 0; u < kTopRUnroll; ++u) {
        const int c4 = base + kThreads * u;
        buf[u] = c4 < n4 ? __ldcs(s4 + c4) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
#pragma unroll
      for (int u = 0; u < kTopRUnroll; ++u) {
        const int c = 4 * (base + kThreads * u);
        if (c < 4 * n4) {
          offer(buf[u].x, c);
          offer(buf[u].y, c + 1);
          offer(buf[u].z, c + 2);
          offer(buf[u].w, c + 3);
        }
      }
    }
    c_scalar = 4 * n4;
  }
  for (int c = c_scalar + tid; c < N; c += kThreads) offer(__ldcs(sr + c), c);

  // R rounds of an argmax over the lanes' list heads; a column appears in one
  // list only, so exactly one lane holds each winner and pops it
  auto warp_merge = [&](float& out_v, int& out_i) {
    out_v = -INFINITY;
    out_i = 0x7fffffff;
    for (int r = 0; r < R; ++r) {
      float bv = v[0];
      int bi = ix[0];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ranks_before(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == r) {
        out_v = bv;
        out_i = bi;
      }
      if (ix[0] == bi && bi != 0x7fffffff) {
#pragma unroll
        for (int i = 0; i + 1 < kMax; ++i) {
          v[i] = v[i + 1];
          ix[i] = ix[i + 1];
        }
        v[kMax - 1] = -INFINITY;
        ix[kMax - 1] = 0x7fffffff;
      }
    }
  };
  float wv;
  int wi;
  warp_merge(wv, wi);
  if (lane < R) {
    s_v[warp][lane] = wv;
    s_i[warp][lane] = wi;
  }
  __syncthreads();
  if (warp != 0) return;
  // warp 0: lane l < 8 walks warp list l (sorted), the others offer nothing
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const bool has = lane < kRecallWarps && i < R;
    v[i] = has ? s_v[lane < kRecallWarps ? lane : 0][i] : -INFINITY;
    ix[i] = has ? s_i[lane < kRecallWarps ? lane : 0][i] : 0x7fffffff;
  }
  float my_v;
  int my_i;
  warp_merge(my_v, my_i);
  // softmax over the R selected scores (slot 0 holds the maximum)
  const float vmax = __shfl_sync(0xffffffffu, my_v, 0);
  const float e = lane < R ? __expf((my_v - vmax) * scale) : 0.f;
  float sum = e;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane < R) {
    idx[(int64_t)row * R + lane] = my_i;
    w[(int64_t)row * R + lane] = e / sum;
  }
}

// out[b, t, :] = sum_r w[row, r] values[idx[row, r], :] for every token t of
// block j (row = b * nq + j).
__global__ void __launch_bounds__(kRecallWarps * 32) recall_gather_kernel(
    const int* __restrict__ idx, const float* __restrict__ w, int R, const __nv_bfloat16* __restrict__ values,
    int64_t ldv, int nv, int D, int T, int L, int nq, __nv_bfloat16* __restrict__ out, int64_t o_sb, int64_t o_st,
    uint32_t* status) {
  __shared__ uint4 vec[32];
  __shared__ int s_idx[32];
  __shared__ float s_w[32];
  const int row = blockIdx.x;
  const int b = row / nq;
  const int j = row % nq;
  const int warp = warp_id();
  const int lane = lane_id();
  const int d0 = blockIdx.y * kRecallSlice + lane * 8;
  if (threadIdx.x < R) {
    int c = idx[(int64_t)row * R + threadIdx.x];
    float wt = w[(int64_t)row * R + threadIdx.x];
    if (c < 0 || c >= nv) {  // not a chunk of the bank: contributes nothing, flagged
      atomicOr(status, kStatusBadLaunch);
      c = 0;
      wt = 0.f;
    }
    s_idx[threadIdx.x] = c;
    s_w[threadIdx.x] = wt;
  }
  __syncthreads();
  if (warp == 0) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (d0 < D) {
      for (int r = 0; r < R; ++r) {
        float f[8];
        unpack8f(__ldg(reinterpret_cast<const uint4*>(values + (int64_t)s_idx[r] * ldv + d0)), f);
        const float wt = s_w[r];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = fmaf(wt, f[c], acc[c]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    vec[lane] = o;
  }
  __syncthreads();
  if (d0 >= D) return;
  const uint4 o = vec[lane];
  const int t0 = j * L;
  const int t1 = min(t0 + L, T);
  __nv_bfloat16* ob = out + (int64_t)b * o_sb + d0;
  for (int t = t0 + warp; t < t1; t += kRecallWarps) __stcs(reinterpret_cast<uint4*>(ob + (int64_t)t * o_st), o);
}

bool al16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_block_mean(const __nv_bfloat16* x, int64_t x_sb, int64_t x_st, int B, int T, int D, int L,
                      __nv_bfloat16* q, int64_t ldq, cudaStream_t stream) {
  if (B <= 0 || T <= 0 || D <= 0 || L <= 0) return set_error(kErrInvalidArgument, "block_mean: empty shape");
  if (D % 8 || x_st % 8 || x_sb % 8 || ldq % 8 || ldq < D || x_st < D || !al16p(x) || !al16p(q))
    return set_error(kErrInvalidArgument,
                     "block_mean: D and strides must be multiples of 8, tensors 16-byte aligned");
  const int nq = (T + L - 1) / L;
  const dim3 grid((unsigned)(B * nq), (unsigned)((D + kRecallSlice - 1) / kRecallSlice));
  block_mean_kernel<<<grid, kRecallWarps * 32, 0, stream>>>(x, x_sb, x_st, T, D, L, nq, q, ldq);
  return check_cuda(cudaGetLastError(), "block_mean launch");
}

int launch_topr(const float* scores, int64_t lds, int M, int N, int R, float scale, int* idx, float* w,
                cudaStream_t stream) {
  if (M <= 0 || N <= 0) return set_error(kErrInvalidArgument, "topr: empty shape");
  if (R < 1 || R > 32) return set_error(kErrUnsupported, "topr: R must be 1..32");
  if (R > N) return set_error(kErrInvalidArgument, "topr: R exceeds the number of chunks");
  if (lds < N) return set_error(kErrInvalidArgument, "topr: row stride smaller than the row");
  const unsigned grid = (unsigned)M;
  if (R <= 4)
    topr_kernel<4><<<grid, kRecallWarps * 32, 0, stream>>>(scores, lds, M, N, R, scale, idx, w);
  else if (R <= 8)
    topr_kernel<8><<<grid, kRecallWarps * 32, 0, stream>>>(scores, lds, M, N, R, scale, idx, w);
  else if (R <= 16)
    topr_kernel<16><<<grid, kRecallWarps * 32, 0, stream>>>(scores, lds, M, N, R, scale, idx, w);
  else
    topr_kernel<32><<<grid, kRecallWarps * 32, 0, stream>>>(scores, lds, M, N, R, scale, idx, w);
  return check_cuda(cudaGetLastError(), "topr launch");
}

int launch_recall_gather(const int* idx, const float* w, int R, const __nv_bfloat16* values, int64_t ldv, int nv,
                         int D, int B, int T, int L, __nv_bfloat16* out, int64_t o_sb, int64_t o_st,
                         cudaStream_t stream) {
  if (B <= 0 || T <= 0 || D <= 0 || L <= 0 || nv <= 0) return set_error(kErrInvalidArgument, "recall_gather: empty shape");
  if (R < 1 || R > 32) return set_error(kErrUnsupported, "recall_gather: R must be 1..32");
  if (D % 8 || ldv % 8 || o_st % 8 || o_sb % 8 || ldv < D || o_st < D || !al16p(values) || !al16p(out))
    return set_error(kErrInvalidArgument,
                     "recall_gather: D and strides must be multiples of 8, tensors 16-byte aligned");
  const int nq = (T + L - 1) / L;
  const dim3 grid((unsigned)(B * nq), (unsigned)((D + kRecallSlice - 1) / kRecallSlice));
  recall_gather_kernel<<<grid, kRecallWarps * 32, 0, stream>>>(idx, w, R, values, ldv, nv, D, T, L, nq, out, o_sb,
                                                                o_st, device_status_word());
  return check_cuda(cudaGetLastError(), "recall_gather launch");
}

}  // namespace fmka
