// On-device split of ggml weight blocks into the GEMV's planes (model load path).
//
// The reference cuts ggml blocks into KURN's split planes on the host with numpy (src/komp/host.py:16-22): Q4_0
// blocks of 18 bytes (f16 d at byte 0, 16 quant bytes at byte 2) and TQ2_0 blocks of 66 bytes (64 quant bytes at
// byte 0, f16 d at byte 64) become WQ = the quant bytes of each row, blocks in order, and WS = the f16 scale bits.
// Here the same cut runs on the GPU on blocks already in device memory (e.g. a GGUF tensor copied up as is), so a
// model's weights are uploaded once in their file layout and split in HBM.
//
// One CTA takes 256 consecutive blocks: it stages their bytes in shared memory with 16-byte loads (256 blocks of 18
// or 66 bytes are a whole number of 16-byte units, so every CTA's range starts 16-byte aligned when the source does),
// then each thread writes its block's quant bytes (16-byte stores) and scale. HBM-bound: reads 18/16 (66/64) of
// the quant bytes, writes them once plus the scales.
#include "b2q_internal.h"

namespace b2q {

template <int NB, int QOFF, int QBYTES, int SOFF>
__global__ void __launch_bounds__(256) split_blocks_kernel(const uint8_t* __restrict__ src, int64_t total,
                                                           int64_t nb, uint8_t* __restrict__ wq, int64_t ldwq,
                                                           int16_t* __restrict__ ws) {
  __shared__ __align__(16) uint8_t stage[256 * NB];
  const int64_t b0 = (int64_t)blockIdx.x * 256;
  const int nblk = (int)min((int64_t)256, total - b0);
  const uint8_t* base = src + b0 * NB;
  const int bytes = nblk * NB;
  const int units = bytes / 16;
  for (int u = threadIdx.x; u < units; u += blockDim.x)
    reinterpret_cast<uint4*>(stage)[u] = reinterpret_cast<const uint4*>(base)[u];
  for (int i = units * 16 + threadIdx.x; i < bytes; i += blockDim.x) stage[i] = base[i];  // tail of the last CTA
  __syncthreads();
  if ((int)threadIdx.x >= nblk) return;
  const int64_t b = b0 + threadIdx.x;
  const int64_t row = b / nb, j = b - row * nb;
  const uint8_t* blk = stage + threadIdx.x * NB;  // 2-byte aligned (NB is even)
  const uint16_t* h = reinterpret_cast<const uint16_t*>(blk + QOFF);
  uint8_t* dst = wq + row * ldwq + j * QBYTES;  // 16-byte aligned (ldwq % 16 == 0, QBYTES % 16 == 0)
#pragma unroll
  for (int q = 0; q < QBYTES / 16; ++q) {
    const uint16_t* p = h + q * 8;
    uint4 v;
    v.x = (uint32_t)p[0] | ((uint32_t)p[1] << 16);
    v.y = (uint32_t)p[2] | ((uint32_t)p[3] << 16);
    v.z = (uint32_t)p[4] | ((uint32_t)p[5] << 16);
    v.w = (uint32_t)p[6] | ((uint32_t)p[7] << 16);
    reinterpret_cast<uint4*>(dst)[q] = v;
  }
  ws[row * nb + j] = *reinterpret_cast<const int16_t*>(blk + SOFF);
}

// Q4_K (144-byte ggml blocks: f16 d, f16 dmin, 12 bytes of packed 6-bit scales and mins, 128 nibble bytes whose
// 32-byte group g holds sub-block 2g in the low and 2g+1 in the high nibbles) -> this backend's planes: per sub-block
// j one 16-byte Q4_0-layout chunk (byte i: value i low, value i + 16 high) and a 20-byte record (d, dmin, then sc_j,
// m_j unpacked). One thread per block, blocks staged in shared memory as above (256 x 144 bytes: 16-byte units).
__global__ void __launch_bounds__(256) split_q4_k_kernel(const uint8_t* __restrict__ src, int64_t total, int64_t nb,
                                                         uint8_t* __restrict__ wq, int64_t ldwq,
                                                         int16_t* __restrict__ ws) {
  __shared__ __align__(16) uint8_t stage[256 * 144];
  const int64_t b0 = (int64_t)blockIdx.x * 256;
  const int nblk = (int)min((int64_t)256, total - b0);
  const uint4* base = reinterpret_cast<const uint4*>(src + b0 * 144);
  for (int u = threadIdx.x; u < nblk * 9; u += blockDim.x) reinterpret_cast<uint4*>(stage)[u] = base[u];
  __syncthreads();
  if ((int)threadIdx.x >= nblk) return;
  const int64_t b = b0 + threadIdx.x;
  const int64_t row = b / nb, j = b - row * nb;
  const uint8_t* blk = stage + threadIdx.x * 144;  // 16-byte aligned
  const uint4* qs = reinterpret_cast<const uint4*>(blk + 16);
  uint4* dst = reinterpret_cast<uint4*>(wq + row * ldwq + j * 128);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint4 a = qs[2 * g], c = qs[2 * g + 1];  // values 0..15 and 16..31 of sub-blocks 2g (low) / 2g+1 (high)
    auto lo = [](uint32_t x, uint32_t y) { return (x & 0x0F0F0F0Fu) | ((y & 0x0F0F0F0Fu) << 4); };
    auto hi = [](uint32_t x, uint32_t y) { return ((x >> 4) & 0x0F0F0F0Fu) | (y & 0xF0F0F0F0u); };
    dst[2 * g] = make_uint4(lo(a.x, c.x), lo(a.y, c.y), lo(a.z, c.z), lo(a.w, c.w));
    dst[2 * g + 1] = make_uint4(hi(a.x, c.x), hi(a.y, c.y), hi(a.z, c.z), hi(a.w, c.w));
  }
  uint8_t rec[20];
  for (int i = 0; i < 4; ++i) rec[i] = blk[i];
  const uint8_t* sc = blk + 4;
  for (int i = 0; i < 4; ++i) {
    rec[4 + 2 * i] = sc[i] & 0x3F;
    rec[5 + 2 * i] = sc[4 + i] & 0x3F;
    rec[12 + 2 * i] = (uint8_t)((sc[8 + i] & 0x0F) | ((sc[i] >> 2) & 0x30));
    rec[13 + 2 * i] = (uint8_t)((sc[8 + i] >> 4) | ((sc[4 + i] >> 2) & 0x30));
  }
  uint8_t* wd = reinterpret_cast<uint8_t*>(ws + (row * nb + j) * 10);  // 4-byte aligned (ws is 16-byte aligned)
  for (int i = 0; i < 20; i += 4)
    *reinterpret_cast<uint32_t*>(wd + i) =
        (uint32_t)rec[i] | ((uint32_t)rec[i + 1] << 8) | ((uint32_t)rec[i + 2] << 16) | ((uint32_t)rec[i + 3] << 24);
}

}  // namespace b2q

using namespace b2q;

extern "C" int b2q_split_blocks(int fmt, const uint8_t* blocks, int64_t n, int64_t k, uint8_t* wq, int64_t ldwq,
                                int16_t* ws, b2q_stream_t stream) {
  const char* who = "b2q_split_blocks";
  if (fmt < 0 || fmt > 4)
    return fail(B2Q_EINVAL, "%s: fmt %d is not Q4_0 (0), TQ2_0 (1), Q8_0 (2), IQ4_NL (3) or Q4_K (4)", who, fmt);
  const int blk = (fmt == 1 || fmt == 4) ? 256 : 32,
            qb = (fmt == 0 || fmt == 3) ? 16 : fmt == 1 ? 64 : fmt == 4 ? 128 : 32;
  if (n < 0 || k < 0) return fail(B2Q_EINVAL, "%s: negative size", who);
  if (k % blk) return fail(B2Q_EINVAL, "%s: k=%lld is not a multiple of the %d-value block", who, (long long)k, blk);
  const int64_t nb = k / blk, total = n * nb;
  if (total == 0) return B2Q_OK;
  if (!blocks || !wq || !ws) return fail(B2Q_EINVAL, "%s: null pointer", who);
  if (ldwq < nb * qb) return fail(B2Q_EINVAL, "%s: ldwq=%lld < %lld quant bytes per row", who, (long long)ldwq,
                                  (long long)(nb * qb));
  if (!aligned(blocks, 16) || !aligned(wq, 16) || (ldwq % 16) || !aligned(ws, 2))
    return fail(B2Q_EALIGN, "%s: blocks and wq must be 16-byte aligned, ldwq %% 16 == 0, ws 2-byte aligned", who);
  if (fmt == 4 && !aligned(ws, 16))
    return fail(B2Q_EALIGN, "%s: Q4_K scale records need ws 16-byte aligned", who);
  const unsigned grid = (unsigned)((total + 255) / 256);
  if (fmt == 4)  // Q4_K: 144-byte blocks -> regrouped nibbles and 20-byte scale records
    split_q4_k_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  else if (fmt == 0 || fmt == 3)  // Q4_0 and IQ4_NL: 18-byte blocks, f16 d then 16 nibble bytes
    split_blocks_kernel<18, 2, 16, 0><<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  else if (fmt == 1)
    split_blocks_kernel<66, 0, 64, 64><<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  else  // Q8_0: 34-byte blocks, f16 d then 32 int8 values
    split_blocks_kernel<34, 2, 32, 0><<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  return after_launch("split_blocks");
}
