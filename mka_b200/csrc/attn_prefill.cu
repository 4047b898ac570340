// Causal flash-attention forward (prefill) on tcgen05 tensor cores, head_dim 128,
// GQA, bottom-right causal alignment (query i sees keys <= i + Tk - Tq), with the
// log-sum-exp of every row as a second output.
//
// Reference semantics: the causal attention of the FastMKA forward
// (F.scaled_dot_product_attention at mka/layers/fastmka.py:134,157 and
// mka/hf/attention.py:142; the explicit masked softmax at fastmka.py:166-174 and
// hf/attention.py:188-193; fastmka_attn at mka/cuda/fastmka_attn.cu:51-131, which
// uses the same Tk - Tq causal offset). GQA is handled by indexing the shared
// K/V head instead of materialising _repeat_kv (hf/attention.py:28-33,128-129).
//
// One CTA per (256-query block, query head): two 128-row Q tiles share every
// K/V tile. Warp roles (12 warps, 3 warpgroups):
//   warp 0      TMA producer: Q0, Q1 once, then K and V tiles (128 keys) into a
//               two-stage shared-memory ring (128-byte swizzle)
//   warp 1      TMEM allocator (512 columns: S0 | S1 | O0 | O1), then the MMA
//               issuer: S_i = Q_i K_j^T, and O_i += P_i V_j with P read straight
//               from TMEM (written there over S_i), interleaved so one tile's
//               GEMMs run while the other tile's softmax runs
//   warps 2,3   idle (complete the first warpgroup)
//   warps 4..7  softmax of Q tile 0, warps 8..11 softmax of Q tile 1: thread =
//               query row; reads its S row from TMEM once into registers (216
//               per thread through setmaxnreg), causal mask on diagonal
//               tiles, running max m and sum z, writes P (bf16) back over S,
//               rescales O in TMEM only when the max grew by more than 2^8
//               (exact: the final 1/z uses the same stale max). One pair
//               of exponentials in sixteen runs on the FMA pipe (exp2_poly2)
//               to relieve the special-function unit. At the end the
//               warpgroup normalises O and writes O and LSE.
// KV tiles past a Q tile's causal limit are neither loaded nor multiplied.
#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

constexpr int kBM = 128;        // rows per Q tile
constexpr int kQTiles = 2;      // Q tiles per CTA
constexpr int kBlockRows = kBM * kQTiles;
constexpr int kBN = 128;        // keys per K/V tile
constexpr int kHeadDim = 128;
constexpr int kKS = 2;          // K/V ring stages
constexpr int kThreads = 384;  // 3 warpgroups
// Register split (setmaxnreg, issued at the top of each role's branch so that
// ptxas allocates each role with its own budget): the producer/MMA warpgroup
// gives registers to the two softmax warpgroups, which keep their whole S row
// (128 scores) in registers from the max pass to the exponentials instead of
// reading it from TMEM again (1.770 against 1.795 ms at batch 4 x 8192; 64/216
// is the smallest control share ptxas compiles without spills). The launch
// holds kThreads x (registers ptxas assigned); the split must fit in it or
// setmaxnreg.inc would wait forever, so the launcher checks kMinLaunchRegs
// against the compiled kernel first.
#ifndef FMKA_ATTN_REG_SPLIT
#define FMKA_ATTN_REG_SPLIT 1
#endif
constexpr int kRegsControl = 64;
constexpr int kRegsSoftmax = 216;
constexpr int kMinLaunchRegs = (128 * kRegsControl + 256 * kRegsSoftmax + kThreads - 1) / kThreads;
constexpr int kTileBytes = 128 * 128 * 2;   // 32 KB
constexpr int kHalfBytes = kTileBytes / 2;  // one 64-column swizzle box
constexpr int kSmemBytes = kTileBytes * (kQTiles + 2 * kKS) + 1024 + 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// One pair in every FMKA_POLY_EVERY pairs of exponentials runs on the FMA pipe.
// Measured (batch 4 x 8192 and 1 x 32768, 28/4 heads, same box, two runs each):
// one in 4: 1054 / 1169 TFLOP/s, one in 8: 1041-1051 / 1165-1176, one in 16:
// 1081 / 1210, none: 1085 / 1201-1211. The softmax step is bound by its
// latency, not by the MUFU's throughput, and the polynomial is the longer path.
#ifndef FMKA_POLY_EVERY
#define FMKA_POLY_EVERY 16
#endif
// L2 policies on the TMA loads (Q evict-first, K/V evict-last) and streaming O
// stores, so that K/V stay in L2 for the other query heads and blocks.
#ifndef FMKA_ATTN_L2_HINTS
#define FMKA_ATTN_L2_HINTS 1
#endif
// Pack P to bf16 with integer rounding (ALU pipe) instead of cvt (XU pipe).
#ifndef FMKA_PACK_ALU
#define FMKA_PACK_ALU 0
#endif

// bf16x2 of two non-negative finite floats, rounded to nearest (ties away
// from zero) on the integer ALU: add half an ulp of bf16, keep the high halves.
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float lo, float hi) {
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  return __byte_perm(a, b, 0x7632);
}

struct AttnParams {
  int B, Hq, Hkv, Tq, Tk;
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;  // O[b, t, h, :]
  int64_t o_sb, o_st, o_sh;
  // o_rows_per_dst > 0: query rows [j * o_rows_per_dst, (j + 1) * o_rows_per_dst)
  // of every sequence go to o_dst.p[j] (row t - j * o_rows_per_dst there), a
  // local or peer-mapped buffer with the same strides; p.o is unused.
  int o_rows_per_dst;
  PeerPtrs o_dst;
  float* lse;        // lse[b, h, t] (may be null)
  int64_t lse_sb, lse_sh;
  int n_qblocks;
  uint32_t* status;
};

// 2^x for a pair on the FMA pipe: Cody-Waite split x = n + f with n = round(x),
// f in [-1/2, 1/2]; 2^f from a degree-3 polynomial fitted here by minimax on the
// relative error (max 8.4e-5, well below the bf16 rounding of P); 2^n added to
// the exponent bits. Inputs below -126 return 2^-126.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = fadd2(x, make_float2(12582912.0f, 12582912.0f));
  const float2 r = fadd2(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = ffma2(r, make_float2(-1.0f, -1.0f), x);
  float2 p = ffma2(make_float2(0.055212993174791336f, 0.055212993174791336f), f,
                   make_float2(0.24271413683891296f, 0.24271413683891296f));
  p = ffma2(p, f, make_float2(0.6932621598243713f, 0.6932621598243713f));
  p = ffma2(p, f, make_float2(0.999919593334198f, 0.999919593334198f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ int kv_tiles_for(int r0, int Tq, int Tk, int offset, int causal) {
  if (r0 >= Tq) return 0;
  if (!causal) return (Tk + kBN - 1) / kBN;
  int last = r0 + kBM - 1 + offset;
  if (last > Tk - 1) last = Tk - 1;
  return last < 0 ? 0 : last / kBN + 1;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                // [2][32 KB]
  uint8_t* sK = smem + kQTiles * kTileBytes;         // [kKS][32 KB]
  uint8_t* sV = sK + kKS * kTileBytes;               // [kKS][32 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kKS * kTileBytes);
  uint64_t* q_full = bars;             // [2]
  uint64_t* k_full = q_full + 2;       // [kKS]
  uint64_t* k_empty = k_full + kKS;    // [kKS]
  uint64_t* v_full = k_empty + kKS;    // [kKS]
  uint64_t* v_empty = v_full + kKS;    // [kKS]
  uint64_t* s_full = v_empty + kKS;    // [2] per Q tile
  uint64_t* p_full = s_full + 2;       // [2] per Q tile
  uint64_t* pv_bar = p_full + 2;       // [2][2]: PV of tile i, kv step j completes pv_bar[2i + (j & 1)]
  uint64_t* o_full = pv_bar + 4;       // [2] the last PV of tile i has completed
  uint64_t* mma_done = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  // ---- block coordinates: the G query heads of one KV head are adjacent,
  // heavy (late) query blocks first ----
  const int G = p.Hq / p.Hkv;
  int idx = blockIdx.x;
  const int g = idx % G;
  idx /= G;
  const int hkv = idx % p.Hkv;
  idx /= p.Hkv;
  const int b = idx % p.B;
  idx /= p.B;
  const int qb = p.n_qblocks - 1 - idx;
  const int hq = hkv * G + g;
  const int q0 = qb * kBlockRows;
  const int offset = p.Tk - p.Tq;
  const int n0 = kv_tiles_for(q0, p.Tq, p.Tk, offset, p.causal);
  const int n1 = kv_tiles_for(q0 + kBM, p.Tq, p.Tk, offset, p.causal);
  const int n_load = n0 > n1 ? n0 : n1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per softmax warp
      mbar_init(&o_full[i], 1);
    }
    for (int s = 0; s < kKS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&pv_bar[i], 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;


  if (warp == 0) {
#if FMKA_ATTN_REG_SPLIT
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
#endif
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const int nt[2] = {n0, n1};
#if FMKA_ATTN_L2_HINTS
      // Q is read by one CTA only; K/V are read again by the other query heads
      // of the group and the other query blocks: keep those in L2
      const uint64_t pol_q = make_l2_policy_evict_first();
      const uint64_t pol_kv = make_l2_policy_evict_last();
#endif
      for (int i = 0; i < kQTiles; ++i) {
        if (nt[i] == 0) continue;
        mbar_arrive_expect_tx(&q_full[i], kTileBytes);
#if FMKA_ATTN_L2_HINTS
        tma_load_4d_hint(sQ + i * kTileBytes, &tmQ, &q_full[i], 0, q0 + i * kBM, hq, b, pol_q);
        tma_load_4d_hint(sQ + i * kTileBytes + kHalfBytes, &tmQ, &q_full[i], 64, q0 + i * kBM, hq, b, pol_q);
#else
        tma_load_4d(sQ + i * kTileBytes, &tmQ, &q_full[i], 0, q0 + i * kBM, hq, b);
        tma_load_4d(sQ + i * kTileBytes + kHalfBytes, &tmQ, &q_full[i], 64, q0 + i * kBM, hq, b);
#endif
      }
      int last_k = -1, last_v = -1;
      for (int j = 0; j < n_load && !*abort_flag; ++j) {
        const int ks = j % kKS;
        const uint32_t ph = (j / kKS) & 1;
        if (!mbar_wait(&k_empty[ks], ph ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
#if FMKA_ATTN_L2_HINTS
        tma_load_4d_hint(sK + ks * kTileBytes, &tmK, &k_full[ks], 0, j * kBN, hkv, b, pol_kv);
        tma_load_4d_hint(sK + ks * kTileBytes + kHalfBytes, &tmK, &k_full[ks], 64, j * kBN, hkv, b, pol_kv);
#else
        tma_load_4d(sK + ks * kTileBytes, &tmK, &k_full[ks], 0, j * kBN, hkv, b);
        tma_load_4d(sK + ks * kTileBytes + kHalfBytes, &tmK, &k_full[ks], 64, j * kBN, hkv, b);
#endif
        last_k = j;
        if (!mbar_wait(&v_empty[ks], ph ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[ks], kTileBytes);
#if FMKA_ATTN_L2_HINTS
        tma_load_4d_hint(sV + ks * kTileBytes, &tmV, &v_full[ks], 0, j * kBN, hkv, b, pol_kv);
        tma_load_4d_hint(sV + ks * kTileBytes + kHalfBytes, &tmV, &v_full[ks], 64, j * kBN, hkv, b, pol_kv);
#else
        tma_load_4d(sV + ks * kTileBytes, &tmV, &v_full[ks], 0, j * kBN, hkv, b);
        tma_load_4d(sV + ks * kTileBytes + kHalfBytes, &tmV, &v_full[ks], 64, j * kBN, hkv, b);
#endif
        last_v = j;
      }
      // Drain: every issued TMA load has landed before teardown (on the normal
      // path the MMA warp has already consumed them all).
      for (int i = 0; i < kQTiles; ++i)
        if (nt[i] > 0) mbar_wait(&q_full[i], 0, p.status);
      for (int j = last_k; j >= 0 && j > last_k - kKS; --j) mbar_wait(&k_full[j % kKS], (j / kKS) & 1, p.status);
      for (int j = last_v; j >= 0 && j > last_v - kKS; --j) mbar_wait(&v_full[j % kKS], (j / kKS) & 1, p.status);
    }
  } else if (warp == 1) {
#if FMKA_ATTN_REG_SPLIT
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
#endif
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_bf16(kBM, kBN, false, false);
      constexpr uint32_t id_pv = make_idesc_bf16(kBM, kHeadDim, false, true);
      const int nt[2] = {n0, n1};
      bool ok = true;
      auto issue_s = [&](int i, int j) {
        if (!ok) return;
        const int ks = j % kKS;
        if (!mbar_wait(&k_full[ks], (j / kKS) & 1, p.status)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + i * kTileBytes);
        const uint32_t k_addr = smem_u32(sK + ks * kTileBytes);
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_ss(d, desc_kmajor_sw128(q_addr + off), desc_kmajor_sw128(k_addr + off), id_s, k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[i]);
      };
      auto issue_pv = [&](int i, int j) {
        if (!ok) return;
        const int vs = j % kKS;
        if (!mbar_wait(&v_full[vs], (j / kKS) & 1, p.status) || !mbar_wait(&p_full[i], j & 1, p.status)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + vs * kTileBytes);
        const uint32_t p_tmem = tmem + i * 128;
        const uint32_t o_tmem = tmem + 256 + i * 128;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          umma_ts(o_tmem, p_tmem + k * 8, desc_mnmajor_sw128(v_addr + k * 2048, kHalfBytes), id_pv,
                  (j > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&pv_bar[2 * i + (j & 1)]);
        if (j == nt[i] - 1) tc_commit(&o_full[i]);
      };
      for (int i = 0; i < kQTiles; ++i)
        if (nt[i] > 0 && !mbar_wait(&q_full[i], 0, p.status)) ok = false;
      if (ok) tc_fence_after();
      for (int i = 0; i < kQTiles; ++i)
        if (nt[i] > 0) issue_s(i, 0);
      if (ok && n_load > 0) tc_commit(&k_empty[0]);
      for (int j = 0; ok && j < n_load; ++j) {
        for (int i = 0; i < kQTiles; ++i) {
          if (j < nt[i]) issue_pv(i, j);
          if (j + 1 < nt[i]) issue_s(i, j + 1);
        }
        if (!ok) break;
        tc_commit(&v_empty[j % kKS]);
        if (j + 1 < n_load) tc_commit(&k_empty[(j + 1) % kKS]);
        if (*abort_flag) ok = false;
      }
      if (!ok) *abort_flag = 1;
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, p.status);
    }
  } else if (warp >= 4) {
#if FMKA_ATTN_REG_SPLIT
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
#endif
    // ------------------------------------------------------------- softmax --
    const int ti = (warp - 4) / 4;  // Q tile of this warpgroup
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const int q = q0 + ti * kBM + r;
    const int n_kv = ti == 0 ? n0 : n1;
    const int qlim = p.causal ? q + offset : p.Tk - 1;  // last visible key
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_col = ti * 128;
    const uint32_t o_col = 256 + ti * 128;
    float m_used = -INFINITY;
    float z = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[ti], j & 1, p.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kbase = j * kBN;
      const bool diag = kbase + kBN - 1 > qlim;  // this tile needs the causal / length mask
      // ---- pass 1: row max over the 128 scores (kept in registers for pass 2) ----
      float mx0;
      uint32_t s[128];
      {
        tmem_ld32(lane_addr + s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tmem_ld32(lane_addr + s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        tmem_ld32(lane_addr + s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
        tmem_ld32(lane_addr + s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
        tmem_wait_ld();
        if (diag) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (kbase + c > qlim) s[c] = 0xFF800000u;  // -inf
        }
        // eight independent chains of three-input maxima
        float mxa[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mxa[a] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; c += 16) {
#pragma unroll
          for (int a = 0; a < 8; ++a) mxa[a] = fmax3(mxa[a], __uint_as_float(s[c + a]), __uint_as_float(s[c + 8 + a]));
        }
        mx0 = fmax3(fmax3(mxa[0], mxa[1], mxa[2]), fmax3(mxa[3], mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7]));
      }
      const float mx = mx0 * p.scale_log2;
      float alpha = 1.f;
      // Warp-uniform decision (tcgen05.ld/st are warp-collective): when any row
      // needs a larger max, every row of the warp moves its max up to
      // max(m_used, mx), which is always valid for the online softmax.
      if (__any_sync(0xffffffffu, mx > m_used + kRescaleThreshold)) {
        const float m_new = fmaxf(m_used, mx);
        alpha = (m_new == m_used) ? 1.f : fast_exp2(m_used - m_new);  // 0 on the first tile
        if (j > 0) {
          // O holds P_0..P_{j-1} V: wait for the last PV, then rescale it.
          if (!__all_sync(0xffffffffu,
                          mbar_wait(&pv_bar[2 * ti + ((j - 1) & 1)], ((j - 1) >> 1) & 1, p.status))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t o[32];
            tmem_ld32(lane_addr + o_col + c4 * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(lane_addr + o_col + c4 * 32, o);
          }
        }
        m_used = m_new;
      }
      // ---- pass 2: P = 2^(s * scale - m) chunk by chunk; P chunk c (16 packed
      // columns) lands on columns already consumed ----
      const float msub = (m_used == -INFINITY) ? 0.f : m_used;
      const float2 sl2 = make_float2(p.scale_log2, p.scale_log2);
      const float2 nm2 = make_float2(-msub, -msub);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const uint32_t* sc = s + 32 * ch;  // masked in pass 1
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float2 xx = ffma2(make_float2(__uint_as_float(sc[2 * c]), __uint_as_float(sc[2 * c + 1])), sl2, nm2);
          float2 pp;
          if ((c % FMKA_POLY_EVERY) == FMKA_POLY_EVERY - 1) {
            pp = exp2_poly2(xx);
          } else {
            pp.x = fast_exp2(xx.x);
            pp.y = fast_exp2(xx.y);
          }
          acc[c & 3] = fadd2(acc[c & 3], pp);
#if FMKA_PACK_ALU
          pk[c] = pack_bf16x2_alu(pp.x, pp.y);
#else
          pk[c] = pack_bf16x2(pp.x, pp.y);
#endif
        }
        tmem_st16(lane_addr + s_col + 16 * ch, pk);
      }
      const float2 a01 = fadd2(acc[0], acc[1]);
      const float2 a23 = fadd2(acc[2], acc[3]);
      const float2 asum = fadd2(a01, a23);
      z = z * alpha + (asum.x + asum.y);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();  // every lane's P store has completed (wait::st) before the warp's arrival
      if (lane == 0) mbar_arrive(&p_full[ti]);
    }
    if (!ok) *abort_flag = 1;
    // ---- epilogue: O / z and LSE ----
    if (n_kv > 0) {
      if (__all_sync(0xffffffffu, ok && mbar_wait(&o_full[ti], 0, p.status))) {
        tc_fence_after();
        const float inv = z > 0.f ? 1.f / z : 0.f;
        const bool row_ok = q < p.Tq;
        __nv_bfloat16* obase = p.o;
        int qo = q;
        if (p.o_rows_per_dst > 0 && row_ok) {
          const int j = q / p.o_rows_per_dst;
          obase = p.o_dst.p[j];
          qo = q - j * p.o_rows_per_dst;
        }
        __nv_bfloat16* dst = obase + (int64_t)b * p.o_sb + (int64_t)qo * p.o_st + (int64_t)hq * p.o_sh;
#pragma unroll 1
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t o[32];
          tmem_ld32(lane_addr + o_col + c4 * 32, o);
          tmem_wait_ld();
          if (row_ok) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
#if FMKA_ATTN_L2_HINTS
              if (p.o_rows_per_dst > 0) d4[v] = w;  // peer stores: plain
              else __stcs(d4 + v, w);               // written once, read by the next kernel
#else
              d4[v] = w;
#endif
            }
          }
        }
        if (row_ok && p.lse != nullptr) {
          p.lse[(int64_t)b * p.lse_sb + (int64_t)hq * p.lse_sh + q] = m_used * 0.69314718055994531f + __logf(z);
        }
        // Rows stored into peer memory are ordered before whatever this GPU
        // does next (the barrier kernel that announces them to the peers).
        if (p.o_rows_per_dst > 0) __threadfence_system();
      } else {
        *abort_flag = 1;
      }
    }
  }
#if FMKA_ATTN_REG_SPLIT
  else {  // warps 2 and 3 complete the first warpgroup's release
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
  }
#endif

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_attn_prefill(const __nv_bfloat16* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                        const __nv_bfloat16* k, const __nv_bfloat16* v, int64_t kv_sb, int64_t kv_sh,
                        int64_t kv_st, __nv_bfloat16* o, int64_t o_sb, int64_t o_st, int64_t o_sh, float* lse,
                        int64_t lse_sb, int64_t lse_sh, int B, int Hq, int Hkv, int Tq, int Tk, int head_dim,
                        int causal, float scale, cudaStream_t stream, const PeerPtrs* o_dst, int n_dst,
                        int rows_per_dst) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Tq <= 0 || Tk <= 0)
    return set_error(kErrInvalidArgument, "attn_prefill: empty shape");
  const bool scatter = o_dst != nullptr;
  if (scatter) {
    if (n_dst < 1 || n_dst > kMaxPeers || rows_per_dst <= 0 || (int64_t)rows_per_dst * n_dst < Tq)
      return set_error(kErrInvalidArgument, "attn_prefill: scatter destinations do not cover the query rows");
    for (int j = 0; j < n_dst; ++j)
      if (o_dst->p[j] == nullptr || (reinterpret_cast<uintptr_t>(o_dst->p[j]) & 15u))
        return set_error(kErrInvalidArgument, "attn_prefill: scatter destinations must be 16-byte aligned");
    o = o_dst->p[0];
  }
  if (head_dim != kHeadDim) return set_error(kErrUnsupported, "attn_prefill: head_dim must be 128");
  if (Hq % Hkv != 0) return set_error(kErrInvalidArgument, "attn_prefill: query heads must be a multiple of kv heads");
  if (causal && Tk < Tq) return set_error(kErrInvalidArgument, "attn_prefill: causal attention needs Tk >= Tq");
  if ((q_st % 8) || (q_sh % 8) || (q_sb % 8) || (kv_st % 8) || (kv_sh % 8) || (kv_sb % 8) || (o_st % 8) ||
      (o_sh % 8) || (o_sb % 8))
    return set_error(kErrInvalidArgument, "attn_prefill: strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return set_error(kErrInvalidArgument, "attn_prefill: tensors must be 16-byte aligned");

  CUtensorMap tmQ, tmK, tmV;
  const uint32_t box[4] = {64, 128, 1, 1};
  {
    uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)Tq, (uint64_t)Hq, (uint64_t)B};
    uint64_t strides[3] = {(uint64_t)q_st * 2, (uint64_t)q_sh * 2, (uint64_t)q_sb * 2};
    int rc = make_tmap_bf16(&tmQ, q, 4, dims, strides, box, true);
    if (rc) return rc;
  }
  {
    uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)Tk, (uint64_t)Hkv, (uint64_t)B};
    uint64_t strides[3] = {(uint64_t)kv_st * 2, (uint64_t)kv_sh * 2, (uint64_t)kv_sb * 2};
    int rc = make_tmap_bf16(&tmK, k, 4, dims, strides, box, true);
    if (rc) return rc;
    rc = make_tmap_bf16(&tmV, v, 4, dims, strides, box, true);
    if (rc) return rc;
  }
  AttnParams p;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Tq = Tq;
  p.Tk = Tk;
  p.causal = causal;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_sb = o_sb;
  p.o_st = o_st;
  p.o_sh = o_sh;
  p.o_rows_per_dst = scatter ? rows_per_dst : 0;
  for (int j = 0; j < kMaxPeers; ++j) p.o_dst.p[j] = (scatter && j < n_dst) ? o_dst->p[j] : nullptr;
  p.lse = lse;
  p.lse_sb = lse_sb;
  p.lse_sh = lse_sh;
  p.n_qblocks = (Tq + kBlockRows - 1) / kBlockRows;
  p.status = device_status_word();
  const int64_t grid = (int64_t)p.n_qblocks * B * Hq;
  if (grid > 0x7FFFFFFF) return set_error(kErrUnsupported, "attn_prefill: problem too large");
  int rc = check_cuda(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes),
                      "attn_prefill attr");
  if (rc) return rc;
  static int launch_regs = 0;
  if (launch_regs == 0) {
    cudaFuncAttributes fa;
    rc = check_cuda(cudaFuncGetAttributes(&fa, attn_prefill_kernel), "attn_prefill attributes");
    if (rc) return rc;
    launch_regs = fa.numRegs;
  }
  if (FMKA_ATTN_REG_SPLIT && launch_regs < kMinLaunchRegs)
    return set_error(kErrUnsupported, "attn_prefill: compiled register count too small for the warpgroup register split");
  attn_prefill_kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, p);
  return check_cuda(cudaGetLastError(), "attn_prefill launch");
}

}  // namespace fmka
