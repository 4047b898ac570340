// Single-token decode attention over a cached K/V, split along the keys.
//
// Reference semantics: the decode branch of the FastMKA forward, where the new
// token attends to cat(past, new) with the explicit masked softmax
// (mka/layers/fastmka.py:102-106,166-174; mka/hf/attention.py:121-129,188-193)
// or the fastmka_attn kernel (mka/cuda/fastmka_attn.cu:51-131). With one query
// the causal mask admits every cached key. GQA shares each K/V row among the
// G = Hq / Hkv query heads of its group instead of materialising _repeat_kv.
//
// The step is HBM-bound: every K and V byte of the cache is read exactly once.
// One CTA handles (batch, kv head, key split):
//   warp 4      TMA producer: 64-key K and V tiles (two 64x64 128-byte-swizzled
//               boxes each) into a 3-stage ring
//   warps 0..3  consumers: warp w takes keys [16w, 16w+16) of every tile; the
//               G <= 16 query heads of the group form the 16 rows of an
//               m16n8k16 MMA (S = Q K^T, then O += P V with P kept in
//               registers), with an online softmax per head row
// At the end the four warps' (max, sum, O) are merged in shared memory; a split
// either writes the final O and LSE (one split) or its normalised partial O and
// log2-sum-exp for attn_decode_combine_kernel.
#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

constexpr int kHeadDim = 128;
constexpr int kTileKeys = 64;
constexpr int kStages = 3;
constexpr int kBoxBytes = 64 * 64 * 2;        // 8 KB
constexpr int kTileBytes = 2 * kBoxBytes;     // 16 KB (64 keys x 128 dims)
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kRingBytes = kStages * 2 * kTileBytes;  // K and V
constexpr int kCombineBytes = kConsumerWarps * (16 * kHeadDim + 32) * 4;
constexpr int kSmemBytes = (kRingBytes > kCombineBytes ? kRingBytes : kCombineBytes) + 1024 + 256;

struct DecodeParams {
  const __nv_bfloat16* q;  // q[b, h, :]
  int64_t q_sb, q_sh;
  int B, Hq, Hkv, Tk;
  float scale_log2;
  int num_splits, keys_per_split;  // keys_per_split is a multiple of kTileKeys
  __nv_bfloat16* o;  // final output o[b, h, :] (one split)
  int64_t o_sb, o_sh;
  float* lse;  // lse[b, h] (one split; may be null)
  int64_t lse_sb;
  float* part_o;    // [B, Hq, num_splits, Dh] normalised partial outputs
  float* part_lse;  // [B, Hq, num_splits] log2-sum-exp (scaled scores)
  uint32_t* status;
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` (0..15 across 128 dims) of key row `row`
// inside a tile stored as two 128-byte-swizzled {64 dims x 64 keys} boxes.
__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
  return (chunk >> 3) * kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

__global__ void __launch_bounds__(kThreads, 2)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + kStages * kTileBytes;
  const int ring_or_combine = kRingBytes > kCombineBytes ? kRingBytes : kCombineBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ring_or_combine);
  uint64_t* full = bars;              // [kStages]
  uint64_t* empty = bars + kStages;   // [kStages]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStages);

  const int warp = warp_id();
  const int lane = lane_id();
  const int G = p.Hq / p.Hkv;

  int idx = blockIdx.x;
  const int split = idx % p.num_splits;
  idx /= p.num_splits;
  const int hkv = idx % p.Hkv;
  const int b = idx / p.Hkv;
  const int k_begin = split * p.keys_per_split;
  int k_end = k_begin + p.keys_per_split;
  if (k_end > p.Tk) k_end = p.Tk;
  const int n_tiles = k_end > k_begin ? (k_end - k_begin + kTileKeys - 1) / kTileKeys : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int last = -1;
      for (int i = 0; i < n_tiles && !*abort_flag; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        const int key0 = k_begin + i * kTileKeys;
        mbar_arrive_expect_tx(&full[s], 2 * kTileBytes);
        tma_load_4d(sK + s * kTileBytes, &tmK, &full[s], 0, key0, hkv, b);
        tma_load_4d(sK + s * kTileBytes + kBoxBytes, &tmK, &full[s], 64, key0, hkv, b);
        tma_load_4d(sV + s * kTileBytes, &tmV, &full[s], 0, key0, hkv, b);
        tma_load_4d(sV + s * kTileBytes + kBoxBytes, &tmV, &full[s], 64, key0, hkv, b);
        last = i;
      }
      for (int i = last; i >= 0 && i > last - kStages; --i) mbar_wait(&full[i % kStages], (i / kStages) & 1, p.status);
    }
    __syncwarp();
    __syncthreads();  // pairs with the consumers' barrier before the merge
    __syncthreads();  // pairs with the consumers' barrier after the merge
    return;
  }

  // ------------------------------------------------------------ consumers --
  const int r_lo = lane >> 2;          // head rows r_lo and r_lo + 8
  const int kq = (lane & 3) * 2;       // key / dim pair within an 8-wide group
  // Q fragments (rows >= G are zero).
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qb = p.q + (int64_t)b * p.q_sb + (int64_t)(hkv * G) * p.q_sh;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d0 = ks * 16 + kq;
      auto ld2 = [&](int row, int d) -> uint32_t {
        if (row >= G) return 0u;
        return *reinterpret_cast<const uint32_t*>(qb + (int64_t)row * p.q_sh + d);
      };
      qa[ks][0] = ld2(r_lo, d0);
      qa[ks][1] = ld2(r_lo + 8, d0);
      qa[ks][2] = ld2(r_lo, d0 + 8);
      qa[ks][3] = ld2(r_lo + 8, d0 + 8);
    }
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY;  // running max (log2 domain)
  float l_lo = 0.f, l_hi = 0.f;              // per-thread partial sums

  const uint32_t k_base = smem_u32(sK);
  const uint32_t v_base = smem_u32(sV);
  const int mrow = lane & 7;   // row inside an 8x8 matrix for ldmatrix addressing
  const int msel = lane >> 3;  // which of the four matrices this lane addresses

  for (int i = 0; i < n_tiles; ++i) {
    const int s = i % kStages;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (i / kStages) & 1, p.status))) {
      *abort_flag = 1;
      break;
    }
    const uint32_t kt = k_base + s * kTileBytes;
    const uint32_t vt = v_base + s * kTileBytes;
    const int key0 = k_begin + i * kTileKeys + warp * 16;  // first key of this warp

    // ---- S = Q K^T : 16 heads x 16 keys ----
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int row = warp * 16 + nt * 8 + mrow;
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kt + swz_off(row, s4 * 4 + msel), b0, b1, b2, b3);
        mma_bf16_16816(sc[nt], qa[2 * s4], b0, b1);
        mma_bf16_16816(sc[nt], qa[2 * s4 + 1], b2, b3);
      }
    }
    // ---- mask keys past the split / cache end, online softmax ----
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int key = key0 + nt * 8 + kq + c;
        if (key >= k_end) {
          sc[nt][c] = -INFINITY;
          sc[nt][2 + c] = -INFINITY;
        }
        sc[nt][c] *= p.scale_log2;
        sc[nt][2 + c] *= p.scale_log2;
        mx_lo = fmaxf(mx_lo, sc[nt][c]);
        mx_hi = fmaxf(mx_hi, sc[nt][2 + c]);
      }
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo);
    const float mn_hi = fmaxf(m_hi, mx_hi);
    const float sub_lo = mn_lo == -INFINITY ? 0.f : mn_lo;
    const float sub_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
    const float al_lo = fast_exp2(m_lo - sub_lo);
    const float al_hi = fast_exp2(m_hi - sub_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      pr[nt][0] = fast_exp2(sc[nt][0] - sub_lo);
      pr[nt][1] = fast_exp2(sc[nt][1] - sub_lo);
      pr[nt][2] = fast_exp2(sc[nt][2] - sub_hi);
      pr[nt][3] = fast_exp2(sc[nt][3] - sub_hi);
    }
    l_lo = l_lo * al_lo + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l_hi = l_hi * al_hi + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= al_lo;
      o[dt][1] *= al_lo;
      o[dt][2] *= al_hi;
      o[dt][3] *= al_hi;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(pr[0][0], pr[0][1]);
    pa[1] = pack_bf16x2(pr[0][2], pr[0][3]);
    pa[2] = pack_bf16x2(pr[1][0], pr[1][1]);
    pa[3] = pack_bf16x2(pr[1][2], pr[1][3]);
    // ---- O += P V : 16 heads x 128 dims ----
    {
      // matrices: (keys 0-7, dims dt), (keys 8-15, dims dt), (keys 0-7, dt+1), (keys 8-15, dt+1)
      const int row = warp * 16 + (msel & 1) * 8 + mrow;
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vt + swz_off(row, dp * 2 + (msel >> 1)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pa, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- merge the four warps ----
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  __syncthreads();  // every warp is done with the ring (producer included)
  float* cO = reinterpret_cast<float*>(smem);                         // [4][16][128]
  float* cML = cO + kConsumerWarps * 16 * kHeadDim;                    // [4][16][2]
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = dt * 8 + kq;
    float* w0 = cO + (warp * 16 + r_lo) * kHeadDim + d;
    float* w1 = cO + (warp * 16 + r_lo + 8) * kHeadDim + d;
    w0[0] = o[dt][0];
    w0[1] = o[dt][1];
    w1[0] = o[dt][2];
    w1[1] = o[dt][3];
  }
  if ((lane & 3) == 0) {
    cML[(warp * 16 + r_lo) * 2 + 0] = m_lo;
    cML[(warp * 16 + r_lo) * 2 + 1] = l_lo;
    cML[(warp * 16 + r_lo + 8) * 2 + 0] = m_hi;
    cML[(warp * 16 + r_lo + 8) * 2 + 1] = l_hi;
  }
  __syncthreads();
  // 128 consumer threads: thread t handles head row t / 8, dims [16 (t % 8), +16)
  {
    const int t = threadIdx.x;
    const int row = t >> 3;
    const int dseg = (t & 7) * 16;
    if (row < G) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cML[(w * 16 + row) * 2]);
      const float Ms = M == -INFINITY ? 0.f : M;
      float L = 0.f;
      float wts[kConsumerWarps];
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        wts[w] = fast_exp2(cML[(w * 16 + row) * 2] - Ms);
        L += wts[w] * cML[(w * 16 + row) * 2 + 1];
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) v += wts[w] * cO[(w * 16 + row) * kHeadDim + dseg + j];
        acc[j] = v * inv;
      }
      const int hq = hkv * G + row;
      // log2-sum-exp of the scaled scores of this split
      const float lse2 = (L > 0.f) ? Ms + __log2f(L) : -INFINITY;
      if (p.num_splits == 1) {
        uint4* dst = reinterpret_cast<uint4*>(p.o + (int64_t)b * p.o_sb + (int64_t)hq * p.o_sh + dseg);
        uint4 w0, w1;
        w0.x = pack_bf16x2(acc[0], acc[1]);
        w0.y = pack_bf16x2(acc[2], acc[3]);
        w0.z = pack_bf16x2(acc[4], acc[5]);
        w0.w = pack_bf16x2(acc[6], acc[7]);
        w1.x = pack_bf16x2(acc[8], acc[9]);
        w1.y = pack_bf16x2(acc[10], acc[11]);
        w1.z = pack_bf16x2(acc[12], acc[13]);
        w1.w = pack_bf16x2(acc[14], acc[15]);
        dst[0] = w0;
        dst[1] = w1;
        if (dseg == 0 && p.lse != nullptr) p.lse[(int64_t)b * p.lse_sb + hq] = lse2 * 0.69314718055994531f;
      } else {
        const int64_t rec = ((int64_t)b * p.Hq + hq) * p.num_splits + split;
        float4* dst = reinterpret_cast<float4*>(p.part_o + rec * kHeadDim + dseg);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        if (dseg == 0) p.part_lse[rec] = lse2;
      }
    }
  }
}

// Merges the per-split partial outputs: one warp per (batch, query head).
__global__ void attn_decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                           int B, int Hq, int num_splits, __nv_bfloat16* __restrict__ o,
                                           int64_t o_sb, int64_t o_sh, float* __restrict__ lse, int64_t lse_sb) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= B * Hq) return;
  const int b = gw / Hq;
  const int h = gw % Hq;
  const float* pl = part_lse + (int64_t)gw * num_splits;
  float M = -INFINITY;
  for (int s = 0; s < num_splits; ++s) M = fmaxf(M, pl[s]);
  const float Ms = M == -INFINITY ? 0.f : M;
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < num_splits; ++s) {
    const float w = fast_exp2(pl[s] - Ms);
    L += w;
    const float4 v = reinterpret_cast<const float4*>(part_o + ((int64_t)gw * num_splits + s) * kHeadDim)[lane];
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint2 packed;
  packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  reinterpret_cast<uint2*>(o + (int64_t)b * o_sb + (int64_t)h * o_sh)[lane] = packed;
  if (lane == 0 && lse != nullptr) lse[(int64_t)b * lse_sb + h] = (Ms + __log2f(L)) * 0.69314718055994531f;
}

}  // namespace

size_t attn_decode_workspace_bytes(int B, int Hq, int num_splits) {
  if (num_splits <= 1) return 0;
  return (size_t)B * Hq * num_splits * (kHeadDim + 1) * sizeof(float);
}

// Splits so that the grid fills whole waves of (2 CTAs x SMs) as closely as
// possible while every split keeps at least 4 tiles of keys.
int attn_decode_default_splits(int B, int Hkv, int Tk, int num_sms) {
  const int pairs = B * Hkv;
  const int max_by_len = (Tk + 4 * kTileKeys - 1) / (4 * kTileKeys);
  const int slots = 2 * num_sms;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= 64 && s <= max_by_len; ++s) {
    const long ctas = (long)pairs * s;
    const long waves = (ctas + slots - 1) / slots;
    const double eff = (double)ctas / (double)(waves * slots);
    // prefer fewer splits unless the wave efficiency improves noticeably
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
    if (ctas >= 8L * slots) break;
  }
  return best;
}

// Final split count for a requested one (<= 0: device default); keys per split
// rounded up to whole tiles.
int attn_decode_plan(int B, int Hkv, int Tk, int requested, int* keys_per_split_out) {
  int s = requested > 0 ? requested : attn_decode_default_splits(B, Hkv, Tk, num_sms_current_device());
  if (s > (Tk + kTileKeys - 1) / kTileKeys) s = (Tk + kTileKeys - 1) / kTileKeys;
  if (s < 1) s = 1;
  int kps = (Tk + s - 1) / s;
  kps = (kps + kTileKeys - 1) / kTileKeys * kTileKeys;
  s = (Tk + kps - 1) / kps;
  if (keys_per_split_out) *keys_per_split_out = kps;
  return s;
}

int launch_attn_decode(const __nv_bfloat16* q, int64_t q_sb, int64_t q_sh, const __nv_bfloat16* k,
                       const __nv_bfloat16* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, __nv_bfloat16* o,
                       int64_t o_sb, int64_t o_sh, float* lse, int64_t lse_sb, int B, int Hq, int Hkv, int Tk,
                       int head_dim, float scale, int num_splits, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Tk <= 0) return set_error(kErrInvalidArgument, "attn_decode: empty shape");
  if (head_dim != kHeadDim) return set_error(kErrUnsupported, "attn_decode: head_dim must be 128");
  if (Hq % Hkv != 0) return set_error(kErrInvalidArgument, "attn_decode: query heads must be a multiple of kv heads");
  if (Hq / Hkv > 16) return set_error(kErrUnsupported, "attn_decode: at most 16 query heads per kv head");
  if ((q_sh % 2) || (q_sb % 2) || (kv_st % 8) || (kv_sh % 8) || (kv_sb % 8) || (o_sh % 8) || (o_sb % 8))
    return set_error(kErrInvalidArgument, "attn_decode: unsupported strides");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15u)
    return set_error(kErrInvalidArgument, "attn_decode: tensors must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(q) & 3u) return set_error(kErrInvalidArgument, "attn_decode: q must be 4-byte aligned");
  int keys_per_split = 0;
  num_splits = attn_decode_plan(B, Hkv, Tk, num_splits, &keys_per_split);
  const size_t need = attn_decode_workspace_bytes(B, Hq, num_splits);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(kErrWorkspace, "attn_decode: workspace too small (need " + std::to_string(need) + " bytes)");
  if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 15u))
    return set_error(kErrInvalidArgument, "attn_decode: workspace must be 16-byte aligned");

  CUtensorMap tmK, tmV;
  const uint32_t box[4] = {64, (uint32_t)kTileKeys, 1, 1};
  uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)Tk, (uint64_t)Hkv, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)kv_st * 2, (uint64_t)kv_sh * 2, (uint64_t)kv_sb * 2};
  int rc = make_tmap_bf16(&tmK, k, 4, dims, strides, box, true);
  if (rc) return rc;
  rc = make_tmap_bf16(&tmV, v, 4, dims, strides, box, true);
  if (rc) return rc;

  DecodeParams p;
  p.q = q;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Tk = Tk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.num_splits = num_splits;
  p.keys_per_split = keys_per_split;
  p.o = o;
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.lse = lse;
  p.lse_sb = lse_sb;
  p.part_o = static_cast<float*>(workspace);
  p.part_lse = p.part_o + (size_t)B * Hq * num_splits * kHeadDim;
  p.status = device_status_word();
  rc = check_cuda(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                  "attn_decode attr");
  if (rc) return rc;
  const int64_t grid = (int64_t)B * Hkv * num_splits;
  attn_decode_kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(tmK, tmV, p);
  rc = check_cuda(cudaGetLastError(), "attn_decode launch");
  if (rc) return rc;
  if (num_splits > 1) {
    const int warps = B * Hq;
    const int threads = 256;
    const int blocks = (warps * 32 + threads - 1) / threads;
    attn_decode_combine_kernel<<<blocks, threads, 0, stream>>>(p.part_o, p.part_lse, B, Hq, num_splits, o, o_sb,
                                                               o_sh, lse, lse_sb);
    rc = check_cuda(cudaGetLastError(), "attn_decode_combine launch");
  }
  return rc;
}

}  // namespace fmka
