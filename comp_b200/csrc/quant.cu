// Standalone activation quantizers (q8_0, q8_K) and the test probes (dp4a, Q4_0/TQ2_0 decode).
//
// The quantizers are memory-trivial (a [4][14336] f32 activation is 229 KB): one pass, fully coalesced, grid-stride.
// The same device functions quantize inside the fused GEMV prologue, so both paths give the same bytes. They take part
// in programmatic dependent launch: each waits for the preceding grid, then at once lets the next grid (a GEMV)
// launch, whose CTAs start streaming weights while the activations are being quantized.
#include "b2q_device.cuh"
#include "b2q_internal.h"

namespace b2q {

// 8 lanes per 32-value block; a lane holds 4 consecutive values (one float4).
__global__ void __launch_bounds__(256) quant_q8_0_kernel(const float* __restrict__ x, int64_t ldx,
                                                         int8_t* __restrict__ xq, float* __restrict__ xd, int64_t M,
                                                         int64_t K) {
  pdl_wait_then_trigger();
  const int64_t nblk = K / 32;
  const int64_t total = M * nblk;
  const int sub = threadIdx.x & 7;
  // a warp covers 4 consecutive blocks per iteration; the loop bound is warp-uniform (shuffles need the full warp)
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t nwarp = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t base = gwarp * 4; base < total; base += nwarp * 4) {
    const int64_t g = base + ((threadIdx.x & 31) >> 3);
    const bool ok = g < total;
    const int64_t m = ok ? g / nblk : 0, b = ok ? g % nblk : 0;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) v = *reinterpret_cast<const float4*>(x + m * ldx + b * 32 + sub * 4);
    float d;
    const uint32_t q = q8_0_quant4(v, &d);
    if (ok) {
      *reinterpret_cast<uint32_t*>(xq + m * K + b * 32 + sub * 4) = q;
      if (sub == 0) xd[m * nblk + b] = q8_0_stored_scale(d);
    }
  }
}

// One warp per 256-value block; lane l holds values 8l..8l+7 (two float4).
__global__ void __launch_bounds__(256) quant_q8_K_kernel(const float* __restrict__ x, int64_t ldx,
                                                         int8_t* __restrict__ xq, float* __restrict__ xd,
                                                         int16_t* __restrict__ bsums, int64_t M, int64_t K) {
  pdl_wait_then_trigger();
  const int64_t nblk = K / 256;
  const int64_t total = M * nblk;
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); g < total; g += stride) {
    const int64_t m = g / nblk, b = g % nblk;
    const float* src = x + m * ldx + b * 256 + lane * 8;
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 c = *reinterpret_cast<const float4*>(src + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    uint32_t qlo, qhi;
    const float d = q8_K_quant8(v, lane, &qlo, &qhi);
    *reinterpret_cast<uint2*>(xq + m * K + b * 256 + lane * 8) = make_uint2(qlo, qhi);
    if (lane == 0) xd[m * nblk + b] = d;
    if (bsums) {
      int s = bytesum(qlo) + bytesum(qhi);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      if ((lane & 1) == 0) bsums[(m * nblk + b) * 16 + (lane >> 1)] = (int16_t)s;
    }
  }
}

__global__ void probe_dp4a_kernel(const int32_t* a, const int32_t* b, const int32_t* c, int32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = dp4a_ss(a[i], b[i], c[i]);
}

// [R][16] bytes -> [R][32] values in natural order: value i = low nibble of byte i, value 16+i = high nibble.
__global__ void decode_q4_0_kernel(const uint8_t* wq, int32_t* out, int64_t R) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= R * 16) return;
  const int64_t r = t / 16;
  const int i = (int)(t % 16);
  const uint8_t q = wq[r * 16 + i];
  out[r * 32 + i] = (int32_t)(q & 15) - 8;
  out[r * 32 + 16 + i] = (int32_t)(q >> 4) - 8;
}

// [R][64] bytes -> [R][256] values: byte h*32+i holds values h*128 + j*32 + i at bits 2j.
__global__ void decode_tq2_0_kernel(const uint8_t* wq, int32_t* out, int64_t R) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= R * 64) return;
  const int64_t r = t / 64;
  const int c = (int)(t % 64);
  const uint8_t q = wq[r * 64 + c];
  const int v0 = (c / 32) * 128 + c % 32;
#pragma unroll
  for (int j = 0; j < 4; ++j) out[r * 256 + v0 + j * 32] = (int32_t)((q >> (2 * j)) & 3) - 1;
}

static int grid_for(int64_t work_items, int per_cta) {
  DeviceInfo di;
  int sms = (device_info(&di) == B2Q_OK) ? di.sms : 148;
  int64_t g = (work_items + per_cta - 1) / per_cta;
  const int64_t cap = (int64_t)sms * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

static int check_quant_args(const char* who, const float* x, int64_t ldx, const int8_t* xq, const float* xd, int64_t M,
                            int64_t K, int blk) {
  if (M < 0 || K < 0) return fail(B2Q_EINVAL, "%s: negative size M=%lld K=%lld", who, (long long)M, (long long)K);
  if (K % blk) return fail(B2Q_EINVAL, "%s: K=%lld is not a multiple of the %d-value block", who, (long long)K, blk);
  if (M == 0 || K == 0) return B2Q_OK;  // nothing to quantize: no pointer is touched
  if (!x || !xq || !xd) return fail(B2Q_EINVAL, "%s: null pointer", who);
  if (ldx < K) return fail(B2Q_EINVAL, "%s: ldx=%lld < K=%lld", who, (long long)ldx, (long long)K);
  if (!aligned(x, 16) || (ldx % 4)) return fail(B2Q_EALIGN, "%s: x must be 16-byte aligned with ldx %% 4 == 0", who);
  if (!aligned(xq, 16)) return fail(B2Q_EALIGN, "%s: xq must be 16-byte aligned", who);
  if (!aligned(xd, 4)) return fail(B2Q_EALIGN, "%s: xd must be 4-byte aligned", who);
  return B2Q_OK;
}

}  // namespace b2q

using namespace b2q;

extern "C" {

int b2q_quant_q8_0(const float* x, int64_t ldx, int8_t* xq, float* xd, int64_t M, int64_t K, b2q_stream_t stream) {
  int rc = check_quant_args("b2q_quant_q8_0", x, ldx, xq, xd, M, K, 32);
  if (rc) return rc;
  if (M == 0 || K == 0) return B2Q_OK;
  const int64_t blocks = M * (K / 32);
  launch_maybe_pdl(quant_q8_0_kernel, dim3(grid_for(blocks, 32)), dim3(256), 0, (cudaStream_t)stream, x, ldx, xq, xd,
                   M, K);
  return after_launch("quant_q8_0");
}

int b2q_quant_q8_K(const float* x, int64_t ldx, int8_t* xq, float* xd, int16_t* bsums, int64_t M, int64_t K,
                   b2q_stream_t stream) {
  int rc = check_quant_args("b2q_quant_q8_K", x, ldx, xq, xd, M, K, 256);
  if (rc) return rc;
  if (bsums && !aligned(bsums, 4)) return fail(B2Q_EALIGN, "b2q_quant_q8_K: bsums must be 4-byte aligned");
  if (M == 0 || K == 0) return B2Q_OK;
  const int64_t blocks = M * (K / 256);
  launch_maybe_pdl(quant_q8_K_kernel, dim3(grid_for(blocks, 8)), dim3(256), 0, (cudaStream_t)stream, x, ldx, xq, xd,
                   bsums, M, K);
  return after_launch("quant_q8_K");
}

int b2q_probe_dp4a(const int32_t* a, const int32_t* b, const int32_t* c, int32_t* out, int64_t n,
                   b2q_stream_t stream) {
  if (!a || !b || !c || !out || n < 0) return fail(B2Q_EINVAL, "b2q_probe_dp4a: bad arguments");
  if (n == 0) return B2Q_OK;
  probe_dp4a_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a, b, c, out, n);
  return after_launch("probe_dp4a");
}

int b2q_decode_q4_0(const uint8_t* wq, int32_t* out, int64_t R, b2q_stream_t stream) {
  if (!wq || !out || R < 0) return fail(B2Q_EINVAL, "b2q_decode_q4_0: bad arguments");
  if (R == 0) return B2Q_OK;
  decode_q4_0_kernel<<<(unsigned)((R * 16 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(wq, out, R);
  return after_launch("decode_q4_0");
}

int b2q_decode_tq2_0(const uint8_t* wq, int32_t* out, int64_t R, b2q_stream_t stream) {
  if (!wq || !out || R < 0) return fail(B2Q_EINVAL, "b2q_decode_tq2_0: bad arguments");
  if (R == 0) return B2Q_OK;
  decode_tq2_0_kernel<<<(unsigned)((R * 64 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(wq, out, R);
  return after_launch("decode_tq2_0");
}

}  // extern "C"
