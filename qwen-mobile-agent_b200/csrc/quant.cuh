// quant.cuh -- Q8_K activation quantization as a warp-level device routine,
// shared by the standalone kernel and the fused layer kernels.
#pragma once
#include "common.cuh"

namespace qma {

// One warp quantizes one 256-lane block: reference quantize_row_q8k
// (q8k.c:34-85).  Lane l owns lanes 8l..8l+7 of the block.
//   xd = amax / 127 (1 when the block is all zero), inv = 1 / xd (IEEE),
//   xq = clamp(round_half_away(x * inv), -127, 127), xsum = sum of xq per 16.
// Bit-identical to the reference: max is exact, the divisions are IEEE
// (this file must not be built with fast-math), roundf rounds half away
// from zero like FCVTAS, and the 16-lane sums are exact integers.
__device__ __forceinline__ void q8k_block_warp_q(const float v[8], int lane, int8_t *xq_blk,
                                                 float *xd_blk, int16_t *xsum_blk, int q[8],
                                                 float &scale) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = warp_max(amax);
    const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / s;
    scale = s;
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int iv = static_cast<int>(roundf(__fmul_rn(v[i], inv)));
        iv = iv > 127 ? 127 : (iv < -127 ? -127 : iv);
        q[i] = iv;
        sum += iv;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    uint2 packed;
    packed.x = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((q[3] & 0xff) << 24);
    packed.y = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((q[7] & 0xff) << 24);
    *reinterpret_cast<uint2 *>(xq_blk + lane * 8) = packed;
    if ((lane & 1) == 0) xsum_blk[lane >> 1] = static_cast<int16_t>(sum);
    if (lane == 0) *xd_blk = s;
}

__device__ __forceinline__ void q8k_block_warp(const float v[8], int lane, int8_t *xq_blk,
                                               float *xd_blk, int16_t *xsum_blk) {
    int q[8];
    float s;
    q8k_block_warp_q(v, lane, xq_blk, xd_blk, xsum_blk, q, s);
}

}  // namespace qma
