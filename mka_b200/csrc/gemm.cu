// Persistent tcgen05 GEMM for the FastMKA projections:
//   C[M, N] = A[M, K] * B[N, K]^T        (A = activations, B = nn.Linear weight)
//
// One CTA per SM walks the output tiles (BM = 128 rows x BN columns). Warp roles:
//   warp 0      TMA producer: A/B K-slices (64 bf16 = one 128-byte swizzle row)
//               into a STAGES-deep shared-memory ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16)
//               into a double-buffered fp32 accumulator in TMEM
//   warp 2      TMEM allocator
//   warps 4..7  epilogue: tcgen05.ld of the accumulator rows (thread i <-> row i),
//               then one of three fused epilogues:
//                 row-major     bias + bf16 store
//                 heads         bias + optional rotate-half RoPE + store straight
//                               into the [B, H, T, Dh] head-split layout
//                 router        bias + SiLU/GELU + dot with the router's second
//                               layer, accumulated into per-token gate logits
// The accumulator is double-buffered so the epilogue of tile i overlaps the
// main loop of tile i+1. With at least two 128-row blocks and 256-wide tiles,
// a CTA-pair kernel (2-SM MMA, 256 x 256 tiles, half the B tile per CTA)
// runs instead; both share the epilogue.
//
// Replaces the nn.Linear calls of the reference FastMKA forward
// (mka/layers/fastmka.py:79,91,98-99,176; mka/hf/attention.py:95,104,110-111,195).
#include <cstdlib>

#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 256;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == 0) return v / (1.0f + __expf(-v));             // SiLU
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));  // GELU (erf form)
}

// Stores 32 fp32 values (held as bits in r) as bf16 to dst; `nvalid` limits
// the columns written (16-byte vector stores when all 32 fit and dst is aligned).
__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const uint32_t (&r)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]), __uint_as_float(r[q * 8 + 1]));
      w.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]), __uint_as_float(r[q * 8 + 3]));
      w.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]), __uint_as_float(r[q * 8 + 5]));
      w.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]), __uint_as_float(r[q * 8 + 7]));
      d4[q] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nvalid) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
  }
}

// 32 fp32 values of one row (the first nvalid of them).
__device__ __forceinline__ void store_row32_f32(float* dst, const uint32_t (&r)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      d4[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                          __uint_as_float(r[4 * q + 3]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nvalid) dst[j] = __uint_as_float(r[j]);
  }
}

// Fused epilogue of one accumulator tile for the calling thread's row `m` (a
// warp's lanes hold 32 consecutive rows): columns n0 .. n0+BN-1 of the output
// from TMEM at acc_addr (this warp's lane quarter, the tile's first column).
template <int BN>
__device__ __forceinline__ void gemm_epilogue_tile(const GemmParams& p, int m, bool row_ok, int n0,
                                                   uint32_t acc_addr) {
  const GemmSeg& sg = (n0 >= p.n_split) ? p.seg[1] : p.seg[0];

  if (sg.kind == kSegRowMajorF32) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(acc_addr + c * 32, r);
      tmem_wait_ld();
      const int n = n0 + c * 32;
      if (row_ok && n < sg.n_end) store_row32_f32(sg.out_f32 + (int64_t)m * sg.ld + (n - sg.n_begin), r, sg.n_end - n);
    }
  } else if (sg.kind == kSegRowMajor) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(acc_addr + c * 32, r);
      tmem_wait_ld();
      const int n = n0 + c * 32;
      if (sg.bias != nullptr) {
        if (n + 32 <= sg.n_end) {
          const float4* b4 = reinterpret_cast<const float4*>(sg.bias + (n - sg.n_begin));
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = __ldg(b4 + q);
            r[4 * q + 0] = __float_as_uint(__uint_as_float(r[4 * q + 0]) + bb.x);
            r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + bb.y);
            r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + bb.z);
            r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + bb.w);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < sg.n_end) r[j] = __float_as_uint(__uint_as_float(r[j]) + __ldg(sg.bias + (n + j - sg.n_begin)));
        }
      }
      if (row_ok && n < sg.n_end) {
        store_row32(sg.out + (int64_t)m * sg.ld + (n - sg.n_begin), r, sg.n_end - n);
      }
    }
  } else if (sg.kind == kSegHeads) {
    const int b = row_ok ? m / sg.T : 0;
    const int t = row_ok ? m % sg.T : 0;
    const bool rope = sg.rope_cos != nullptr;
    const int64_t rope_off = (int64_t)b * sg.rope_sb + (int64_t)t * sg.rope_st;
    __nv_bfloat16* dst_row = sg.out + (int64_t)b * sg.s_b + (int64_t)(t + sg.t_offset) * sg.s_t;
    // 16-column chunks of the first half of every head (dims d) paired with
    // the same chunk of the second half (dims d + 64); the RoPE table slice
    // is loaded once per chunk and shared by the tile's heads.
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float cs1[16], sn1[16], cs2[16], sn2[16];
      if (rope && row_ok) {
        const float4* c4a = reinterpret_cast<const float4*>(sg.rope_cos + rope_off + c * 16);
        const float4* s4a = reinterpret_cast<const float4*>(sg.rope_sin + rope_off + c * 16);
        const float4* c4b = reinterpret_cast<const float4*>(sg.rope_cos + rope_off + 64 + c * 16);
        const float4* s4b = reinterpret_cast<const float4*>(sg.rope_sin + rope_off + 64 + c * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 a0 = __ldg(c4a + q), a1 = __ldg(s4a + q), a2 = __ldg(c4b + q), a3 = __ldg(s4b + q);
          cs1[4 * q] = a0.x; cs1[4 * q + 1] = a0.y; cs1[4 * q + 2] = a0.z; cs1[4 * q + 3] = a0.w;
          sn1[4 * q] = a1.x; sn1[4 * q + 1] = a1.y; sn1[4 * q + 2] = a1.z; sn1[4 * q + 3] = a1.w;
          cs2[4 * q] = a2.x; cs2[4 * q + 1] = a2.y; cs2[4 * q + 2] = a2.z; cs2[4 * q + 3] = a2.w;
          sn2[4 * q] = a3.x; sn2[4 * q + 1] = a3.y; sn2[4 * q + 2] = a3.z; sn2[4 * q + 3] = a3.w;
        }
      }
#pragma unroll
      for (int hh = 0; hh < BN / 128; ++hh) {
        uint32_t r1[16], r2[16];
        tmem_ld16(acc_addr + hh * 128 + c * 16, r1);
        tmem_ld16(acc_addr + hh * 128 + 64 + c * 16, r2);
        tmem_wait_ld();
        const int nl_head = n0 - sg.n_begin + hh * 128;
        const bool in_range = (n0 + hh * 128) < sg.n_end;
        if (sg.bias != nullptr && in_range) {
          const float4* ba = reinterpret_cast<const float4*>(sg.bias + nl_head + c * 16);
          const float4* bb = reinterpret_cast<const float4*>(sg.bias + nl_head + 64 + c * 16);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 x = __ldg(ba + q), y = __ldg(bb + q);
            r1[4 * q] = __float_as_uint(__uint_as_float(r1[4 * q]) + x.x);
            r1[4 * q + 1] = __float_as_uint(__uint_as_float(r1[4 * q + 1]) + x.y);
            r1[4 * q + 2] = __float_as_uint(__uint_as_float(r1[4 * q + 2]) + x.z);
            r1[4 * q + 3] = __float_as_uint(__uint_as_float(r1[4 * q + 3]) + x.w);
            r2[4 * q] = __float_as_uint(__uint_as_float(r2[4 * q]) + y.x);
            r2[4 * q + 1] = __float_as_uint(__uint_as_float(r2[4 * q + 1]) + y.y);
            r2[4 * q + 2] = __float_as_uint(__uint_as_float(r2[4 * q + 2]) + y.z);
            r2[4 * q + 3] = __float_as_uint(__uint_as_float(r2[4 * q + 3]) + y.w);
          }
        }
        uint32_t o1[8], o2[8];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          float a0 = __uint_as_float(r1[j]), a1 = __uint_as_float(r1[j + 1]);
          float b0 = __uint_as_float(r2[j]), b1 = __uint_as_float(r2[j + 1]);
          if (rope) {
            const float ra0 = a0 * cs1[j] - b0 * sn1[j];
            const float ra1 = a1 * cs1[j + 1] - b1 * sn1[j + 1];
            const float rb0 = b0 * cs2[j] + a0 * sn2[j];
            const float rb1 = b1 * cs2[j + 1] + a1 * sn2[j + 1];
            a0 = ra0; a1 = ra1; b0 = rb0; b1 = rb1;
          }
          o1[j / 2] = pack_bf16x2(a0, a1);
          o2[j / 2] = pack_bf16x2(b0, b1);
        }
        if (row_ok && in_range) {
          __nv_bfloat16* dst = dst_row + (int64_t)(nl_head / 128) * sg.s_h;
          uint4* d1 = reinterpret_cast<uint4*>(dst + c * 16);
          uint4* d2 = reinterpret_cast<uint4*>(dst + 64 + c * 16);
          d1[0] = make_uint4(o1[0], o1[1], o1[2], o1[3]);
          d1[1] = make_uint4(o1[4], o1[5], o1[6], o1[7]);
          d2[0] = make_uint4(o2[0], o2[1], o2[2], o2[3]);
          d2[1] = make_uint4(o2[4], o2[5], o2[6], o2[7]);
        }
      }
    }
  } else if (sg.kind == kSegSwiGLU) {
    // Tile columns n0 .. n0+127 are gate rows and n0+128 .. n0+255 the up rows
    // of output channels (n0 - n_begin) / 2 .. + 127 (256-wide tiles only).
    if constexpr (BN == 256) {
      const int oc0 = (n0 - sg.n_begin) / 2;
      const bool in_range = n0 < sg.n_end;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t g[32], u[32];
        tmem_ld32(acc_addr + c * 32, g);
        tmem_ld32(acc_addr + 128 + c * 32, u);
        tmem_wait_ld();
        if (row_ok && in_range) {
          const int nl = n0 - sg.n_begin + c * 32;
          uint32_t r[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float gv = __uint_as_float(g[j]);
            float uv = __uint_as_float(u[j]);
            if (sg.bias != nullptr) {
              gv += __ldg(sg.bias + nl + j);
              uv += __ldg(sg.bias + nl + 128 + j);
            }
            r[j] = __float_as_uint(act_fn(gv, 0) * uv);
          }
          store_row32(sg.out + (int64_t)m * sg.ld + oc0 + c * 32, r, 32);
        }
      }
    }
  } else {  // kSegRouter
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    const int R = sg.n_end - sg.n_begin;
    const int L = sg.L;
    const int act = sg.act;
    const float* w2 = sg.w2;
    const float* bias = sg.bias;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int nl = n0 - sg.n_begin + c * 32;
      uint32_t r[32];
      tmem_ld32(acc_addr + c * 32, r);
      tmem_wait_ld();
      if (nl >= R) continue;  // warp-uniform
      if (nl + 32 <= R && (R & 3) == 0) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
          if (bias != nullptr) bb = __ldg(reinterpret_cast<const float4*>(bias + nl) + q);
          const float a0 = act_fn(__uint_as_float(r[4 * q + 0]) + bb.x, act);
          const float a1 = act_fn(__uint_as_float(r[4 * q + 1]) + bb.y, act);
          const float a2 = act_fn(__uint_as_float(r[4 * q + 2]) + bb.z, act);
          const float a3 = act_fn(__uint_as_float(r[4 * q + 3]) + bb.w, act);
#pragma unroll
          for (int l = 0; l < 4; ++l) {
            if (l < L) {
              const float4 w = __ldg(reinterpret_cast<const float4*>(w2 + (int64_t)l * R + nl) + q);
              part[l] += w.x * a0 + w.y * a1 + w.z * a2 + w.w * a3;
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (nl + j < R) {
            float v = __uint_as_float(r[j]);
            if (bias != nullptr) v += __ldg(bias + nl + j);
            const float a = act_fn(v, act);
#pragma unroll
            for (int l = 0; l < 4; ++l)
              if (l < L) part[l] += __ldg(w2 + (int64_t)l * R + nl + j) * a;
          }
        }
      }
    }
    if (row_ok) {
#pragma unroll
      for (int l = 0; l < 4; ++l)
        if (l < L) atomicAdd(sg.logits + (int64_t)m * L + l, part[l]);
    }
  }
}

// Scatter epilogue (p.n_dst > 0) of one accumulator tile for the calling warp's
// 32 rows m_warp0 .. m_warp0 + 31: bias, bf16, and a store of every row into
// each destination buffer (mostly other GPUs' memory through peer mappings).
// The rows pass through the warp's 8 KB staging area in shared memory (32 rows
// x 128 columns, 16-byte units XOR-swizzled by row so that neither side has
// bank conflicts), so that every store instruction writes two whole 256-byte
// row segments instead of 32 scattered 16-byte pieces: full-width writes keep
// the NVLink packets full.
constexpr int kScatterWarpBytes = 32 * 128 * 2;

template <int BN>
__device__ __forceinline__ void gemm_epilogue_scatter(const GemmParams& p, int m_warp0, int n0, uint32_t acc_addr,
                                                      uint4* stage) {
  const int lane = lane_id();
  const float* bias = p.seg[0].bias;
#pragma unroll 1
  for (int h = 0; h < BN / 128; ++h) {
    const int nh = n0 + h * 128;
    if (nh >= p.N) break;  // warp-uniform
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(acc_addr + h * 128 + c * 32, r);
      tmem_wait_ld();
      const int n = nh + c * 32;
      if (bias != nullptr) {
        if (n + 32 <= p.N) {
          const float4* b4 = reinterpret_cast<const float4*>(bias + n);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = __ldg(b4 + q);
            r[4 * q + 0] = __float_as_uint(__uint_as_float(r[4 * q + 0]) + bb.x);
            r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + bb.y);
            r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + bb.z);
            r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + bb.w);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < p.N) r[j] = __float_as_uint(__uint_as_float(r[j]) + __ldg(bias + n + j));
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]), __uint_as_float(r[q * 8 + 1]));
        w.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]), __uint_as_float(r[q * 8 + 3]));
        w.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]), __uint_as_float(r[q * 8 + 5]));
        w.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]), __uint_as_float(r[q * 8 + 7]));
        stage[lane * 16 + ((c * 4 + q) ^ (lane & 7))] = w;
      }
    }
    __syncwarp();
    // Lanes 0-15 store row 2i, lanes 16-31 row 2i + 1, 16 bytes each.
    const int u = lane & 15;
    const bool col_ok = nh + u * 8 < p.N;  // N is a multiple of 8
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int rr = 2 * i + (lane >> 4);
      const int m = m_warp0 + rr;
      const uint4 w = stage[rr * 16 + (u ^ (rr & 7))];
      if (m < p.M && col_ok) {
        const int64_t off = (p.dst_row0 + m) * p.dst_ld + nh + u * 8;
#pragma unroll 1
        for (int k = 0; k < p.n_dst; ++k) *reinterpret_cast<uint4*>(p.dst.p[k] + off) = w;
      }
    }
    __syncwarp();  // the staging area is read before the next half overwrites it
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* mma_done = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        gemm_tile_coords(tile, num_m, num_n, p.raster_group, mb, nb);
        const int m0 = mb * kBM;
        const int n0 = nb * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          if (p.a_kblk > 0)  // A split along K into blocks of a_kblk columns (a gathered buffer)
            tma_load_3d(sA + stage * Cfg::kABytes, &tmA, &full[stage], (kb * kBK) % p.a_kblk, m0,
                        (kb * kBK) / p.a_kblk);
          else
            tma_load_2d(sA + stage * Cfg::kABytes, &tmA, &full[stage], kb * kBK, m0);
          tma_load_2d(sB + stage * Cfg::kBBytes, &tmB, &full[stage], kb * kBK, n0);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: make sure no TMA write is still landing in shared memory when
      // the CTA tears down (they have all completed on the normal path).
      const long pending = issued < S ? issued : S;
      for (long i = 0; i < pending; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.status);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t aphase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            umma_ss(d_tmem, desc_kmajor_sw128(a_addr + k * 32), desc_kmajor_sw128(b_addr + k * 32), idesc,
                    (kb | k) != 0);
          }
          tc_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_commit(&tfull[acc]);
      }
      // All MMAs issued by this thread complete before teardown.
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue --
    const int ew = warp - 4;
    const int row_in_tile = ew * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(ew * 32) << 16);
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aphase, p.status))) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int mb, nb;
      gemm_tile_coords(tile, num_m, num_n, p.raster_group, mb, nb);
      const int m0 = mb * kBM;
      const int n0 = nb * BN;
      const int m = m0 + row_in_tile;
      const bool row_ok = m < p.M;
      gemm_epilogue_tile<BN>(p, m, row_ok, n0, lane_addr + acc * BN);
      tc_fence_before();
      __syncwarp();  // every lane's TMEM reads have completed before the warp's arrival
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs on neighbouring SMs computes
// 256 x 256 tiles with the 2-SM MMA (M = 256, cta_group::2), issued by the
// even CTA. Each CTA loads only its own 128 A rows and its half (128 rows) of
// the B tile, so a stage is 32 KB per CTA instead of 48 KB: a third less
// operand traffic per FLOP and six stages of loads in flight. Each CTA's TMEM
// holds its 128 rows x 256 columns of the accumulator (double-buffered), and
// each CTA runs the same epilogue on its rows.
// Synchronisation: both CTAs' TMA loads complete on the even CTA's `full`
// barrier (the even CTA's producer posts the byte count of both); the MMA's
// commits arrive on `empty` / `tfull` in both CTAs; both CTAs' epilogue warps
// arrive on the even CTA's `tempty` (8 arrivals).
struct PairCfg {
  static constexpr int kBN = 256;
  static constexpr int kHalfN = 128;
  static constexpr int kStages = 6;
  static constexpr int kABytes = kBM * kBK * 2;     // 16 KB
  static constexpr int kBBytes = kHalfN * kBK * 2;  // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * kBN;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
  // With the scatter epilogue: plus the four epilogue warps' staging areas.
  static constexpr int kScatterBytes = 4 * kScatterWarpBytes;
  static constexpr int kSmemBytesScatter = kSmemBytes + kScatterBytes;
};

// KPS k-blocks per pipeline stage. KPS > 1: each operand of a stage is one 3-D
// TMA box of KPS k-blocks over a [K/64][rows][64] view of the row-major matrix
// (A plain row-major, K a multiple of 64), so the producer issues half or a
// quarter as many boxes; the stage ring keeps the same bytes in flight.
template <bool kScatter, int KPS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ GemmParams p) {
  using Cfg = PairCfg;
  static_assert(Cfg::kStages % KPS == 0, "stages group into whole KPS blocks");
  constexpr int S = Cfg::kStages / KPS;
  constexpr int BN = Cfg::kBN;
  constexpr int kA = KPS * Cfg::kABytes;  // A bytes of one stage
  constexpr int kB = KPS * Cfg::kBBytes;  // B bytes of one stage

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kA;
  uint4* sScatter = reinterpret_cast<uint4*>(smem + S * (kA + kB));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * (kA + kB) + (kScatter ? Cfg::kScatterBytes : 0));
  uint64_t* full = bars;               // [S]  used in the even CTA
  uint64_t* empty = bars + S;          // [S]  both CTAs
  uint64_t* tfull = bars + 2 * S;      // [2]  both CTAs
  uint64_t* tempty = bars + 2 * S + 2; // [2]  used in the even CTA
  uint64_t* mma_done = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  const int num_m = (p.M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised and their TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const uint32_t full_even = cluster_addr(&full[0], 0);
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += npairs) {
        int mb, nb;
        gemm_tile_coords(tile, num_m, num_n, p.raster_group, mb, nb);
        const int m0 = mb * (2 * kBM) + (int)rank * kBM;
        const int n0 = nb * BN + (int)rank * Cfg::kHalfN;
        for (int kb = 0; kb < num_kb; kb += KPS) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
            *abort_flag = 1;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (kA + kB));
          const uint32_t fb = full_even + stage * 8;
          if constexpr (KPS > 1) {
            tma_load_3d_pair(sA + stage * kA, &tmA, fb, 0, m0, kb);
            tma_load_3d_pair(sB + stage * kB, &tmB, fb, 0, n0, kb);
          } else {
            if (p.a_kblk > 0)
              tma_load_3d_pair(sA + stage * kA, &tmA, fb, (kb * kBK) % p.a_kblk, m0, (kb * kBK) / p.a_kblk);
            else
              tma_load_2d_pair(sA + stage * kA, &tmA, fb, kb * kBK, m0);
            tma_load_2d_pair(sB + stage * kB, &tmB, fb, kb * kBK, n0);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: the last fills of each stage have been consumed (their MMAs
      // completed, so their loads landed) before the CTA tears down.
      const long pending = issued < S ? issued : S;
      for (long i = 0; i < pending; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&empty[stage], phase, p.status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA (the even CTA issues) --
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(2 * kBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t aphase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; kb += KPS) {
          if (!mbar_wait(&full[stage], phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kA);
          const uint32_t b_addr = smem_u32(sB + stage * kB);
#pragma unroll
          for (int h = 0; h < KPS; ++h) {
            if (kb + h < num_kb) {  // a box past the last k-block was zero-filled and is skipped
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                umma_ss_pair(d_tmem, desc_kmajor_sw128(a_addr + h * Cfg::kABytes + k * 32),
                             desc_kmajor_sw128(b_addr + h * Cfg::kBBytes + k * 32), idesc, ((kb + h) | k) != 0);
              }
            }
          }
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_commit_pair(&tfull[acc], 0x3);
      }
      // All MMAs (and the commits before this one) complete before teardown.
      tc_commit_pair(mma_done, 0x1);
      mbar_wait(mma_done, 0, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue --
    const int ew = warp - 4;
    const int row_in_tile = ew * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(ew * 32) << 16);
    const uint32_t tempty_even = cluster_addr(&tempty[0], 0);
    int it = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++it) {
      const int acc = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aphase, p.status))) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int mb, nb;
      gemm_tile_coords(tile, num_m, num_n, p.raster_group, mb, nb);
      const int m = mb * (2 * kBM) + (int)rank * kBM + row_in_tile;
      const int n0 = nb * BN;
      if constexpr (kScatter)
        gemm_epilogue_scatter<BN>(p, m - lane, n0, lane_addr + acc * BN,
                                  sScatter + ew * (kScatterWarpBytes / 16));
      else
        gemm_epilogue_tile<BN>(p, m, m < p.M, n0, lane_addr + acc * BN);
      tc_fence_before();
      __syncwarp();  // every lane's TMEM reads have completed before the warp's arrival
      if (lane == 0) mbar_arrive_cluster(tempty_even + acc * 8);
    }
    // Stores into peer memory are ordered before whatever this GPU does next
    // (the barrier kernel that announces them to the peers).
    if constexpr (kScatter) __threadfence_system();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no arrival or commit aimed at either CTA is still outstanding
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Split-K on a cluster, for GEMMs whose M fits one 64-row slice (decode).
// Such a GEMM streams the weights; with one CTA per 128-column tile only
// N/128 CTAs pull them. Here a cluster of S (= kSplitMax) CTAs shares each tile: CTA r
// runs the main loop over the r-th slice of K into its own TMEM. After a
// cluster barrier (every main loop and load has finished, so the stage
// buffers are free), CTAs 1..S-1 store their fp32 partial rows into the stage
// buffers of CTA 0 through distributed shared memory; after a second barrier
// CTA 0 adds them to its accumulator in TMEM and runs the fused epilogue once.
// Every warp of every CTA passes both barriers exactly once, on every path.
constexpr int kSplitRows = 64;   // rows of a partial that are exchanged
// Cluster size. Up to 7 partials of 64 x 128 fp32 would fit the 192 KB of
// stages, but measured on the decode projections (M = 64, K = 4096) pairs are
// fastest: 2 CTAs per tile beat 1 by 9-18 %, while 4 and 7 lose to 2 (each
// CTA's pipeline-fill latency and the two cluster barriers outweigh the
// extra streaming CTAs, and clusters of 7 pack poorly into the GPCs).
constexpr int kSplitMax = 2;
// Cluster size with 64-column tiles (row-major outputs). Measured on the
// decode step (M = 64, K = 4096): 64-column tiles in pairs took kv_proj
// (N = 2048) and o_proj (N = 4096) from 0.0229 to 0.0208 ms each; clusters of
// 4 took kv_proj to 0.0189 ms and did not show in the step's time.
#ifndef FMKA_SPLITK_MAX64
#define FMKA_SPLITK_MAX64 2
#endif
constexpr int kSplitMax64 = FMKA_SPLITK_MAX64;
constexpr int split_max_for(int bn) { return bn == 64 ? kSplitMax64 : kSplitMax; }

// KPS k-blocks per stage; KPS > 1 loads each operand of a stage as one 3-D TMA
// box over a [K/64][rows][64] view, as in gemm_pair_kernel.
template <int BN, int KPS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<BN>;
  static_assert(Cfg::kStages % KPS == 0, "stages group into whole KPS blocks");
  constexpr int S = Cfg::kStages / KPS;
  constexpr int kA = KPS * Cfg::kABytes;  // A bytes of one stage
  constexpr int kB = KPS * Cfg::kBBytes;  // B bytes of one stage
  constexpr int kSlotBytes = kSplitRows * BN * 4;  // 32 KB at BN = 128
  static_assert((split_max_for(BN) - 1) * kSlotBytes <= S * (kA + kB), "the partials fit the stage buffers");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * (kA + kB));
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* mma_done = bars + 2 * S + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  uint32_t csize;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int tile = blockIdx.x / (int)csize;  // BN-column tile of this cluster
  const int n0 = tile * BN;
  const int num_kb = (p.K + kBK - 1) / kBK;
  // balanced slices: none is empty while the cluster has at most num_kb CTAs
  const int kb0 = (int)(((long)rank * num_kb) / (int)csize);
  const int kb1 = (int)(((long)(rank + 1) * num_kb) / (int)csize);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  bool have_acc = false;  // epilogue warps: this CTA's partial is complete in TMEM
  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int kb = kb0; kb < kb1 && !*abort_flag; kb += KPS) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], kA + kB);
        if constexpr (KPS > 1) {
          tma_load_3d(sA + stage * kA, &tmA, &full[stage], 0, 0, kb);
          tma_load_3d(sB + stage * kB, &tmB, &full[stage], 0, n0, kb);
        } else {
          if (p.a_kblk > 0)
            tma_load_3d(sA + stage * kA, &tmA, &full[stage], (kb * kBK) % p.a_kblk, 0, (kb * kBK) / p.a_kblk);
          else
            tma_load_2d(sA + stage * kA, &tmA, &full[stage], kb * kBK, 0);
          tma_load_2d(sB + stage * kB, &tmB, &full[stage], kb * kBK, n0);
        }
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      const long pending = issued < S ? issued : S;
      for (long i = 0; i < pending; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.status);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; kb += KPS) {
        if (!mbar_wait(&full[stage], phase, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + stage * kA);
        const uint32_t b_addr = smem_u32(sB + stage * kB);
#pragma unroll
        for (int h = 0; h < KPS; ++h) {
          if (kb + h < kb1) {  // a box past this CTA's last k-block is loaded and skipped
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              umma_ss(tmem_base, desc_kmajor_sw128(a_addr + h * Cfg::kABytes + k * 32),
                      desc_kmajor_sw128(b_addr + h * Cfg::kBBytes + k * 32), idesc,
                      (kb + h > kb0 || k > 0) ? 1u : 0u);
            }
          }
        }
        tc_commit(&empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) *abort_flag = 1;
      tc_commit(tfull);  // also when no MMA ran: the epilogue then sees an error
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, p.status);
    }
  } else if (warp >= 4) {
    const bool done = mbar_wait(tfull, 0, p.status);
    have_acc = __all_sync(0xffffffffu, done && !*abort_flag);
    if (have_acc) tc_fence_after();
  }

  // ---- every main loop and TMA load of the cluster is done ----
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const int ew = warp - 4;
  const int row = ew * 32 + lane;
  const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(ew * 32) << 16);
  if (warp >= 4 && rank != 0 && have_acc && ew < kSplitRows / 32) {
    // partial rows 0..63 into slot rank-1 of CTA 0's stage buffers
    const uint32_t dst = cluster_addr(smem, 0) + (rank - 1) * kSlotBytes + row * BN * 4;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(lane_addr + c * 32, r);
      tmem_wait_ld();
      if (row < p.M) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst + (c * 32 + q * 4) * 4),
                       "r"(r[4 * q]), "r"(r[4 * q + 1]), "r"(r[4 * q + 2]), "r"(r[4 * q + 3])
                       : "memory");
      }
    }
  }
  __syncwarp();
  cluster_sync();  // the partials have landed in CTA 0
  if (warp >= 4 && rank == 0) {
    const bool ok = have_acc;
    if (ok && ew < kSplitRows / 32) {  // warp-uniform: tcgen05.ld/st are warp-collective
      const float* slots = reinterpret_cast<const float*>(smem) + row * BN;
      const int nslots = row < p.M ? (int)csize - 1 : 0;  // per lane: rows past M were never sent
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_addr + c * 32, r);
        tmem_wait_ld();
        for (int sl = 0; sl < nslots; ++sl) {
          const float4* src = reinterpret_cast<const float4*>(slots + sl * (kSlotBytes / 4) + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 v = src[q];
            r[4 * q] = __float_as_uint(__uint_as_float(r[4 * q]) + v.x);
            r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + v.y);
            r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + v.z);
            r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + v.w);
          }
        }
        tmem_st32(lane_addr + c * 32, r);
      }
    }
    tmem_wait_st();
    if (__all_sync(0xffffffffu, ok)) {
      gemm_epilogue_tile<BN>(p, row, row < p.M, n0, lane_addr);
    } else {
      *abort_flag = 1;
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, BN);
  }
}

}  // namespace

int launch_gemm(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb, const GemmParams& p_in,
                int num_sms, cudaStream_t stream) {
  GemmParams p = p_in;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return set_error(kErrInvalidArgument, "gemm: M, N, K must be positive");
  // Tile order. A weight that fits comfortably in L2 (every projection of the
  // attention layer: at most 29 MB) stays there whatever the order, and the
  // tiles go row-major. A larger one would stream from HBM once per row
  // block, so its tiles go in bands of 8 row blocks, each weight tile reused
  // across the band while it is in L2.
  p.raster_group = ((int64_t)p.N * p.K * 2 > (int64_t(64) << 20)) ? 8 : 1;
  if (p.K % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0)
    return set_error(kErrInvalidArgument, "gemm: K and row strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u))
    return set_error(kErrInvalidArgument, "gemm: A and B must be 16-byte aligned");

  // Tile width: 256 when every segment boundary is 256-aligned, else 128.
  int BN = 256;
  if (p.n_split % 256 != 0 && p.n_split < p.N) BN = 128;
  // One row block (decode-sized M): the GEMM streams weights, and narrower
  // tiles double the number of CTAs pulling them. The SwiGLU epilogue needs a
  // tile to hold both halves of a 256-column block.
  const bool swiglu = p.seg[0].kind == kSegSwiGLU;
  if (p.M <= kBM && !swiglu) BN = 128;
  if (swiglu && (p.N % 256 != 0 || p.n_split < p.N || p.seg[0].ld % 8 != 0 ||
                 (reinterpret_cast<uintptr_t>(p.seg[0].out) & 15u)))
    return set_error(kErrInvalidArgument,
                     "gemm: SwiGLU needs N a multiple of 256, one segment, a 16-byte aligned output");
  if (p.n_split % 128 != 0 && p.n_split < p.N)
    return set_error(kErrInvalidArgument, "gemm: segment split must be a multiple of 128 columns");
  // Scatter epilogue: always the CTA-pair kernel with 256-wide tiles.
  const bool scatter = p.n_dst > 0;
  if (scatter) {
    if (p.n_dst > kMaxPeers) return set_error(kErrInvalidArgument, "gemm: at most 8 scatter destinations");
    if (p.N % 8 != 0 || p.dst_ld % 8 != 0 || p.dst_ld < p.N || p.dst_row0 < 0 || p.n_split < p.N)
      return set_error(kErrInvalidArgument, "gemm: scatter needs N and the row stride multiples of 8, one segment");
    for (int k = 0; k < p.n_dst; ++k)
      if (p.dst.p[k] == nullptr || (reinterpret_cast<uintptr_t>(p.dst.p[k]) & 15u))
        return set_error(kErrInvalidArgument, "gemm: scatter destinations must be 16-byte aligned");
    if (num_sms < 2) return set_error(kErrUnsupported, "gemm: scatter needs two SMs");
    BN = 256;
  }
  for (int s = 0; s < 2; ++s) {
    const GemmSeg& g = p.seg[s];
    if (g.n_end <= g.n_begin) continue;
    if (g.kind == kSegHeads && (g.head_dim != 128 || (g.n_end - g.n_begin) % 128 != 0 || g.T <= 0))
      return set_error(kErrUnsupported, "gemm: head-split epilogue needs head_dim 128 and whole heads");
    if (g.kind == kSegRouter && (g.L < 1 || g.L > 4 || g.w2 == nullptr || g.logits == nullptr))
      return set_error(kErrInvalidArgument, "gemm: router epilogue needs 1..4 levels, w2 and logits");
    if ((g.kind == kSegRowMajor || g.kind == kSegRowMajorF32) && (g.ld % 8 != 0))
      return set_error(kErrInvalidArgument, "gemm: output row stride must be a multiple of 8");
    if (g.kind == kSegRowMajorF32 && (g.out_f32 == nullptr || (reinterpret_cast<uintptr_t>(g.out_f32) & 15u)))
      return set_error(kErrInvalidArgument, "gemm: the fp32 output must be 16-byte aligned");
    // an output row must not run into the next one
    if (p.n_dst == 0 && (g.kind == kSegRowMajor || g.kind == kSegRowMajorF32) && g.ld < g.n_end - g.n_begin)
      return set_error(kErrInvalidArgument, "gemm: output row stride is smaller than the row");
    if (g.kind == kSegSwiGLU && g.ld < (g.n_end - g.n_begin) / 2)
      return set_error(kErrInvalidArgument, "gemm: output row stride is smaller than the row");
  }

  CUtensorMap tmA, tmB;
  if (p.a_kblk > 0) {
    // A[m, k] = A_blocks[k / a_kblk][m][k % a_kblk]: blocks of a_kblk columns, rows
    // lda apart inside a block, blocks a_blk_stride elements apart.
    if (p.a_kblk % kBK != 0 || p.K % p.a_kblk != 0 || p.a_blk_stride % 8 != 0)
      return set_error(kErrInvalidArgument, "gemm: K blocks must be multiples of 64 columns that tile K");
    uint64_t dims[3] = {(uint64_t)p.a_kblk, (uint64_t)p.M, (uint64_t)(p.K / p.a_kblk)};
    uint64_t strides[2] = {(uint64_t)lda * 2, (uint64_t)p.a_blk_stride * 2};
    uint32_t box[3] = {kBK, kBM, 1};
    int rc = make_tmap_bf16(&tmA, A, 3, dims, strides, box, true);
    if (rc) return rc;
  } else {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    uint64_t strides[1] = {(uint64_t)lda * 2};
    uint32_t box[2] = {kBK, kBM};
    int rc = make_tmap_bf16(&tmA, A, 2, dims, strides, box, true);
    if (rc) return rc;
  }
  // CTA pairs for 256-wide tiles whenever there are at least two 128-row
  // blocks; FMKA_GEMM_PAIR=0 in the environment selects the one-CTA kernel.
  static const bool pair_enabled = [] {
    const char* e = std::getenv("FMKA_GEMM_PAIR");
    return e == nullptr || e[0] != '0';
  }();
  const bool use_pair = scatter || (pair_enabled && BN == 256 && p.M > kBM && num_sms >= 2);
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    uint64_t strides[1] = {(uint64_t)ldb * 2};
    uint32_t box[2] = {kBK, use_pair ? (uint32_t)PairCfg::kHalfN : (uint32_t)BN};
    int rc = make_tmap_bf16(&tmB, B, 2, dims, strides, box, true);
    if (rc) return rc;
  }

  // Two k-blocks per TMA box (pair and split-K kernels) where A is plain
  // row-major and K is a multiple of 64; FMKA_GEMM_KPS=1 in the environment
  // keeps one box per k-block.
  static const bool kps2_enabled = [] {
    const char* e = std::getenv("FMKA_GEMM_KPS");
    return e == nullptr || e[0] != '1';
  }();
  // Decode-sized M: split K over a cluster of CTAs per 128-column tile;
  // FMKA_GEMM_SPLITK=0 in the environment keeps one CTA per tile.
  static const bool splitk_enabled = [] {
    const char* e = std::getenv("FMKA_GEMM_SPLITK");
    return e == nullptr || e[0] != '0';
  }();
  // Row-major outputs only (no head-split, router or SwiGLU epilogue, which need
  // whole 128-column heads or blocks): 64-column tiles, twice the CTAs streaming
  // the weights (the MMA's N = 64 runs at half rate, which a weight-bound GEMM
  // does not feel). FMKA_GEMM_SPLIT64=0 keeps 128-column tiles.
  static const bool split64_enabled = [] {
    const char* e = std::getenv("FMKA_GEMM_SPLIT64");
    return e == nullptr || e[0] != '0';
  }();
  auto row_major_only = [&]() {
    for (int sg = 0; sg < 2; ++sg) {
      const GemmSeg& g = p.seg[sg];
      if (g.n_end > g.n_begin && g.kind != kSegRowMajor && g.kind != kSegRowMajorF32) return false;
    }
    return true;
  };
  if (!scatter && splitk_enabled && BN == 128 && p.M <= kSplitRows) {
    const int num_kb = (p.K + kBK - 1) / kBK;
    auto cluster_for = [&](int bn) {
      int c = num_sms / ((p.N + bn - 1) / bn);
      if (c > split_max_for(bn)) c = split_max_for(bn);
      if (c > num_kb) c = num_kb;
      return c;
    };
    // 64-column tiles only where they still leave two CTAs per tile
    const int bn = (split64_enabled && row_major_only() && p.n_split >= p.N && cluster_for(64) >= 2) ? 64 : 128;
    const int tiles = (p.N + bn - 1) / bn;
    const int cs = cluster_for(bn);
    if (cs >= 2 && bn == 64) {
      uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
      uint64_t strides[1] = {(uint64_t)ldb * 2};
      uint32_t box[2] = {kBK, 64u};
      int rc = make_tmap_bf16(&tmB, B, 2, dims, strides, box, true);
      if (rc) return rc;
    }
    if (cs >= 2) {
      const int smem = bn == 64 ? GemmCfg<64>::kSmemBytes : GemmCfg<128>::kSmemBytes;
      const bool kps2 = kps2_enabled && p.a_kblk == 0 && p.K % kBK == 0;
      if (kps2) {
        const uint64_t nkb = (uint64_t)(p.K / kBK);
        uint64_t adims[3] = {(uint64_t)kBK, (uint64_t)p.M, nkb};
        uint64_t astr[2] = {(uint64_t)lda * 2, (uint64_t)kBK * 2};
        uint32_t abox[3] = {kBK, kBM, 2};
        int rc = make_tmap_bf16(&tmA, A, 3, adims, astr, abox, true);
        if (rc) return rc;
        uint64_t bdims[3] = {(uint64_t)kBK, (uint64_t)p.N, nkb};
        uint64_t bstr[2] = {(uint64_t)ldb * 2, (uint64_t)kBK * 2};
        uint32_t bbox[3] = {kBK, (uint32_t)bn, 2};
        rc = make_tmap_bf16(&tmB, B, 3, bdims, bstr, bbox, true);
        if (rc) return rc;
      }
      auto kern = bn == 64 ? (kps2 ? gemm_splitk_kernel<64, 2> : gemm_splitk_kernel<64, 1>)
                           : (kps2 ? gemm_splitk_kernel<128, 2> : gemm_splitk_kernel<128, 1>);
      int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                          "gemm split-K attr");
      if (rc) return rc;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(tiles * cs), 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)cs;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      rc = check_cuda(cudaLaunchKernelEx(&cfg, kern, tmA, tmB, p), "gemm split-K launch");
      if (rc) return rc;
      return check_cuda(cudaGetLastError(), "gemm split-K launch");
    }
  }

  if (use_pair) {
    const int tiles = ((p.M + 2 * kBM - 1) / (2 * kBM)) * ((p.N + PairCfg::kBN - 1) / PairCfg::kBN);
    const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
    const int smem = scatter ? PairCfg::kSmemBytesScatter : PairCfg::kSmemBytes;
    if (kps2_enabled && !scatter && p.a_kblk == 0 && p.K % kBK == 0) {
      const int nkb = p.K / kBK;
      CUtensorMap tA3, tB3;
      {
        uint64_t dims[3] = {(uint64_t)kBK, (uint64_t)p.M, (uint64_t)nkb};
        uint64_t strides[2] = {(uint64_t)lda * 2, (uint64_t)kBK * 2};
        uint32_t box[3] = {kBK, kBM, 2};
        int rc = make_tmap_bf16(&tA3, A, 3, dims, strides, box, true);
        if (rc) return rc;
      }
      {
        uint64_t dims[3] = {(uint64_t)kBK, (uint64_t)p.N, (uint64_t)nkb};
        uint64_t strides[2] = {(uint64_t)ldb * 2, (uint64_t)kBK * 2};
        uint32_t box[3] = {kBK, (uint32_t)PairCfg::kHalfN, 2};
        int rc = make_tmap_bf16(&tB3, B, 3, dims, strides, box, true);
        if (rc) return rc;
      }
      auto kern2 = gemm_pair_kernel<false, 2>;
      int rc = check_cuda(cudaFuncSetAttribute(kern2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                          "gemm pair attr");
      if (rc) return rc;
      kern2<<<2 * pairs, kThreads, smem, stream>>>(tA3, tB3, p);
      return check_cuda(cudaGetLastError(), "gemm pair launch");
    }
    auto kern = scatter ? gemm_pair_kernel<true, 1> : gemm_pair_kernel<false, 1>;
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                        "gemm pair attr");
    if (rc) return rc;
    kern<<<2 * pairs, kThreads, smem, stream>>>(tmA, tmB, p);
    return check_cuda(cudaGetLastError(), "gemm pair launch");
  }

  const int num_tiles = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN);
  const int grid = num_tiles < num_sms ? num_tiles : num_sms;
  if (BN == 256) {
    auto k = gemm_tcgen05_kernel<256>;
    const int smem = GemmCfg<256>::kSmemBytes;
    int rc = check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "gemm attr");
    if (rc) return rc;
    k<<<grid, kThreads, smem, stream>>>(tmA, tmB, p);
  } else {
    auto k = gemm_tcgen05_kernel<128>;
    const int smem = GemmCfg<128>::kSmemBytes;
    int rc = check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "gemm attr");
    if (rc) return rc;
    k<<<grid, kThreads, smem, stream>>>(tmA, tmB, p);
  }
  return check_cuda(cudaGetLastError(), "gemm launch");
}

}  // namespace fmka
