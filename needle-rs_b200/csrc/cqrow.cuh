// Device helpers on CQ matrices shared by the kernel files.
#pragma once

#include "kernels.h"
#include "numerics.cuh"

namespace nd {

// (float)(1 / sqrt(128)), the rotation's scale for a 128-wide group
// (quant.rs:71-73, hadamard_scale(128) rounded to f32).
#define ND_HS128 __uint_as_float(0x3db504f3u)

// QMat::row (qlinear.rs:309-323) of one 128-wide group, by a warp: each
// lane's four weights p = 4 lane .. 4 lane + 3, `fvals[code] * norm`, then
// the rotation. The four codes are 4 * width consecutive bits of the group.
__device__ __forceinline__ void cq_group_row(const DevMat& W, size_t row, int g, int lane, float v[4]) {
    const int width = W.width, bpg = 16 * width;
    const uint8_t* c = W.codes + (row * W.groups + g) * bpg;
    const int bit = 4 * width * lane;
    uint32_t w = (uint32_t)c[bit >> 3];
    if (width > 2) w |= (uint32_t)c[(bit >> 3) + 1] << 8;
    w >>= bit & 7;
    const uint32_t mask = (1u << width) - 1;
    float norm = h2f(W.norms[row * W.groups + g]);
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = __fmul_rn(W.fvals[(w >> (width * k)) & mask], norm);
    fwht128_warp(v, lane);
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = __fmul_rn(v[k], ND_HS128);
}

}  // namespace nd
