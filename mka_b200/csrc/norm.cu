// Elementwise work of the decoder layers around the patched self_attn.
//
// RMSNorm in one pass:
//
// transformers' LlamaRMSNorm / Qwen2RMSNorm (the input_layernorm and
// post_attention_layernorm of every decoder layer of the full-model workload)
// runs as a chain of elementwise kernels with fp32 intermediates:
//   h = x.float(); var = mean(h^2); h = h * rsqrt(var + eps); y = w * h.to(bf16)
// For a [65536, 4096] bf16 input that moves about 8 GB. Here one warp owns a
// row: it reads the row once (16-byte loads, the row stays in registers), sums
// the squares in fp32 with warp shuffles, and writes y once, rounding like the
// module does (h to bf16 first, then the bf16 product with the weight).
//
// SiLU product of the MLP: transformers' LlamaMLP computes
// down_proj(act_fn(gate_proj(x)) * up_proj(x)) with the activation and the
// product as two elementwise kernels over [tokens, intermediate] bf16 tensors
// (for 65536 x 14336 that is ~9.4 GB of traffic); here one pass reads g and u
// and writes bf16(bf16(silu(g)) * u), the module's roundings.
#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

constexpr int kNormWarps = 8;
constexpr int kNormMaxD = 8192;                    // 32 lanes x 32 chunks x 8 channels
constexpr int kNormMaxChunks = kNormMaxD / (32 * 8);

template <int kChunks>
__global__ void __launch_bounds__(kNormWarps * 32) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                  const __nv_bfloat16* __restrict__ w, float eps,
                                                                  __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                                  int rows, int D) {
  const int row = blockIdx.x * kNormWarps + warp_id();
  if (row >= rows) return;
  const int lane = lane_id();
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  uint4 v[kChunks];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int d = (c * 32 + lane) * 8;
    v[c] = d < D ? __ldcs(reinterpret_cast<const uint4*>(xr + d)) : make_uint4(0, 0, 0, 0);
    const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = bf16lo_to_f32(u[q]), b = bf16hi_to_f32(u[q]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)D + eps);
  __nv_bfloat16* yr = y + (int64_t)row * ldy;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int d = (c * 32 + lane) * 8;
    if (d >= D) continue;
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + d));
    const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      // h * rsqrt rounded to bf16, then the bf16 product with the weight
      const uint32_t h = pack_bf16x2(bf16lo_to_f32(u[q]) * r, bf16hi_to_f32(u[q]) * r);
      o[q] = pack_bf16x2(bf16lo_to_f32(wu[q]) * bf16lo_to_f32(h), bf16hi_to_f32(wu[q]) * bf16hi_to_f32(h));
    }
    *reinterpret_cast<uint4*>(yr + d) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* g,  // out may be g
                                                     const __nv_bfloat16* __restrict__ u, __nv_bfloat16* out,
                                                     int64_t n8) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 gv = __ldcs(reinterpret_cast<const uint4*>(g) + i);
    const uint4 uv = __ldcs(reinterpret_cast<const uint4*>(u) + i);
    const uint32_t ga[4] = {gv.x, gv.y, gv.z, gv.w};
    const uint32_t ua[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float g0 = bf16lo_to_f32(ga[q]), g1 = bf16hi_to_f32(ga[q]);
      const uint32_t a = pack_bf16x2(g0 / (1.f + __expf(-g0)), g1 / (1.f + __expf(-g1)));
      o[q] = pack_bf16x2(bf16lo_to_f32(a) * bf16lo_to_f32(ua[q]), bf16hi_to_f32(a) * bf16hi_to_f32(ua[q]));
    }
    __stcs(reinterpret_cast<uint4*>(out) + i, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

}  // namespace

int launch_silu_mul(const __nv_bfloat16* g, const __nv_bfloat16* u, __nv_bfloat16* out, int64_t n,
                    cudaStream_t stream) {
  if (n <= 0) return set_error(kErrInvalidArgument, "silu_mul: empty input");
  if (n % 8 != 0) return set_error(kErrUnsupported, "silu_mul: the element count must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return set_error(kErrInvalidArgument, "silu_mul: tensors must be 16-byte aligned");
  const int64_t n8 = n / 8;
  int64_t blocks = (n8 + 255) / 256;
  const int64_t cap = (int64_t)num_sms_current_device() * 8;
  if (blocks > cap) blocks = cap;
  silu_mul_kernel<<<(unsigned)blocks, 256, 0, stream>>>(g, u, out, n8);
  return check_cuda(cudaGetLastError(), "silu_mul launch");
}

int launch_rmsnorm(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* w, float eps, __nv_bfloat16* y,
                   int64_t ldy, int rows, int D, cudaStream_t stream) {
  if (rows <= 0 || D <= 0) return set_error(kErrInvalidArgument, "rmsnorm: empty shape");
  if (D % 8 != 0 || D > kNormMaxD)
    return set_error(kErrUnsupported, "rmsnorm: the row length must be a multiple of 8 and at most 8192");
  if ((ldx % 8) || (ldy % 8) || ldx < D || ldy < D)
    return set_error(kErrInvalidArgument, "rmsnorm: row strides must be multiples of 8 and at least the row length");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return set_error(kErrInvalidArgument, "rmsnorm: tensors must be 16-byte aligned");
  const unsigned grid = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
  const int chunks = (D + 255) / 256;
  if (chunks <= 4)
    rmsnorm_kernel<4><<<grid, kNormWarps * 32, 0, stream>>>(x, ldx, w, eps, y, ldy, rows, D);
  else if (chunks <= 16)
    rmsnorm_kernel<16><<<grid, kNormWarps * 32, 0, stream>>>(x, ldx, w, eps, y, ldy, rows, D);
  else
    rmsnorm_kernel<kNormMaxChunks><<<grid, kNormWarps * 32, 0, stream>>>(x, ldx, w, eps, y, ldy, rows, D);
  return check_cuda(cudaGetLastError(), "rmsnorm launch");
}

}  // namespace fmka
