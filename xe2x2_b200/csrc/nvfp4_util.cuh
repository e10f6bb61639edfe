// nvfp4_util.cuh -- register-level E2M1 decoding shared by the NVFP4 kernels.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "w4_common.cuh"

namespace w4 {

// Four E2M1 nibbles (x bits 0..15, nibble i = bits 4i..4i+3) -> bf16 pairs:
// r01 = (v0, v1), r23 = (v2, v3), low half first.  E2M1 -> bf16 is a register
// lookup: two byte-permutes read the low / high byte of the bf16 pattern of
// |e2m1| from 8-entry tables held in immediates, a third merges the sign bytes.
__device__ __forceinline__ void e2m1x4_to_bf16(uint32_t x, uint32_t &r01, uint32_t &r23) {
    // |e2m1| in bf16: 0, .5, 1, 1.5 | 2, 3, 4, 6
    constexpr uint32_t TL0 = 0xC0800000u, TL1 = 0xC0804000u;  // low bytes
    constexpr uint32_t TH0 = 0x3F3F3F00u, TH1 = 0x40404040u;  // high bytes
    const uint32_t sel = x & 0x7777u;
    const uint32_t L = __byte_perm(TL0, TL1, sel);
    const uint32_t Hp = __byte_perm(TH0, TH1, sel);
    // sign of nibble i -> bit 7 of byte i: nibbles 1,3 have it at bits 7,15 of x,
    // nibbles 0,2 at bits 3,11 (bits 7,15 of x << 4)
    uint32_t sg;
    asm("prmt.b32 %0, %1, %2, 0x1504;" : "=r"(sg) : "r"(x), "r"(x << 4));
    const uint32_t H = lop3_and_or(sg, 0x80808080u, Hp);
    r01 = __byte_perm(L, H, 0x5140);
    r23 = __byte_perm(L, H, 0x7362);
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162 *>(&a),
                               *reinterpret_cast<__nv_bfloat162 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}


}  // namespace w4
