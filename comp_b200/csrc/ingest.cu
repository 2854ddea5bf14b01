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

}  // namespace b2q

using namespace b2q;

extern "C" int b2q_split_blocks(int fmt, const uint8_t* blocks, int64_t n, int64_t k, uint8_t* wq, int64_t ldwq,
                                int16_t* ws, b2q_stream_t stream) {
  const char* who = "b2q_split_blocks";
  if (fmt < 0 || fmt > 3)
    return fail(B2Q_EINVAL, "%s: fmt %d is not Q4_0 (0), TQ2_0 (1), Q8_0 (2) or IQ4_NL (3)", who, fmt);
  const int blk = fmt == 1 ? 256 : 32, qb = (fmt == 0 || fmt == 3) ? 16 : fmt == 1 ? 64 : 32;
  if (n < 0 || k < 0) return fail(B2Q_EINVAL, "%s: negative size", who);
  if (k % blk) return fail(B2Q_EINVAL, "%s: k=%lld is not a multiple of the %d-value block", who, (long long)k, blk);
  const int64_t nb = k / blk, total = n * nb;
  if (total == 0) return B2Q_OK;
  if (!blocks || !wq || !ws) return fail(B2Q_EINVAL, "%s: null pointer", who);
  if (ldwq < nb * qb) return fail(B2Q_EINVAL, "%s: ldwq=%lld < %lld quant bytes per row", who, (long long)ldwq,
                                  (long long)(nb * qb));
  if (!aligned(blocks, 16) || !aligned(wq, 16) || (ldwq % 16) || !aligned(ws, 2))
    return fail(B2Q_EALIGN, "%s: blocks and wq must be 16-byte aligned, ldwq %% 16 == 0, ws 2-byte aligned", who);
  const unsigned grid = (unsigned)((total + 255) / 256);
  if (fmt == 0 || fmt == 3)  // Q4_0 and IQ4_NL: 18-byte blocks, f16 d then 16 nibble bytes
    split_blocks_kernel<18, 2, 16, 0><<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  else if (fmt == 1)
    split_blocks_kernel<66, 0, 64, 64><<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  else  // Q8_0: 34-byte blocks, f16 d then 32 int8 values
    split_blocks_kernel<34, 2, 32, 0><<<grid, 256, 0, (cudaStream_t)stream>>>(blocks, total, nb, wq, ldwq, ws);
  return after_launch("split_blocks");
}
