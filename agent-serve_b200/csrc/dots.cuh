// Row-dot routines shared by the GEMV kernel (gemv.cu) and the persistent decode kernel
// (persist.cu): fp32 activations (shared memory, xpad layout) times GGUF block weights
// (shared memory, native layout), fp32 accumulation.
#pragma once

#include "common.cuh"

namespace tfb {

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// ---- Q8_0 unit dot with the activation held in registers --------------------------------
// One 64-element unit (two 34-byte blocks, 17 aligned words at wp) of one row against the
// lane's 64 activations xr[] (kept in registers for a whole phase, so shared-memory traffic
// is the weights only).  int8 -> fp32 by the exact construction 0x4B0000xx - (2^23 + 128);
// products on the packed fp32x2 pipe with four independent accumulators per block.
// acc += dA * sum(x*qA) + dB * sum(x*qB)  (the block-scale form of src/quant.cpp:266-283).
__device__ __forceinline__ void unit_dot_q8_reg(const uint32_t* wp, const float (&xr)[64], float& acc) {
    const float2 kBias = make_float2(-8388736.0f, -8388736.0f);
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = wp[i];
    const float dA = h2f(w[0]);
    const float dB = h2f(w[8] >> 16);
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] ^= 0x80808080u;
    float2 sA[4], sB[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) sA[r] = sB[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        float qa[4], qb[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int ja = 2 + 4 * g + e, jb = 36 + 4 * g + e;  // bytes of block A / B in the unit
            qa[e] = __int_as_float((int)__byte_perm(w[ja >> 2], 0x4B000000u, 0x7650u | (uint32_t)(ja & 3)));
            qb[e] = __int_as_float((int)__byte_perm(w[jb >> 2], 0x4B000000u, 0x7650u | (uint32_t)(jb & 3)));
        }
        const float2 qa0 = __fadd2_rn(make_float2(qa[0], qa[1]), kBias), qa1 = __fadd2_rn(make_float2(qa[2], qa[3]), kBias);
        const float2 qb0 = __fadd2_rn(make_float2(qb[0], qb[1]), kBias), qb1 = __fadd2_rn(make_float2(qb[2], qb[3]), kBias);
        const int r0 = (2 * g) & 3, r1 = (2 * g + 1) & 3;
        sA[r0] = __ffma2_rn(make_float2(xr[4 * g], xr[4 * g + 1]), qa0, sA[r0]);
        sA[r1] = __ffma2_rn(make_float2(xr[4 * g + 2], xr[4 * g + 3]), qa1, sA[r1]);
        sB[r0] = __ffma2_rn(make_float2(xr[32 + 4 * g], xr[32 + 4 * g + 1]), qb0, sB[r0]);
        sB[r1] = __ffma2_rn(make_float2(xr[32 + 4 * g + 2], xr[32 + 4 * g + 3]), qb1, sB[r1]);
    }
    const float2 a2 = __fadd2_rn(__fadd2_rn(sA[0], sA[1]), __fadd2_rn(sA[2], sA[3]));
    const float2 b2 = __fadd2_rn(__fadd2_rn(sB[0], sB[1]), __fadd2_rn(sB[2], sB[3]));
    acc = fmaf(dA, a2.x + a2.y, acc);
    acc = fmaf(dB, b2.x + b2.y, acc);
}

// ---- Q8_0 exact-integer path ---------------------------------------------------------------
// The activation row is turned into three signed-byte digit planes, once per kernel: each
// 32-element block is scaled by a power of two 2^sh so that its largest magnitude is below
// 2^22, rounded to integers X, and X = x2*2^16 + x1*2^8 + x0 with x0, x1, x2 in [-128, 127].
// The planes use the byte layout of a Q8_0 row (34 bytes per block, 0 at the two scale
// bytes), so a weight word and the plane word at the same offset line up for dp4a and the
// scale bytes meet zeros.  The block sum sum_j q_j*X_j is then exact in int32 (|.| <= 2^19
// per plane), and sum_j q_j*x_j = (sum q*x2 * 2^16 + sum q*x1 * 2^8 + sum q*x0) * 2^-sh.
// Rounding x to 22 significant bits of its block maximum is the only approximation, the same
// size as the fp32 rounding of the products in src/quant.cpp:266-321; the block scale d is
// applied to the block sum as the reference does.  Cost per weight byte: one dp4a per plane
// and word, against the PRMT/FADD/FFMA conversion chain of the fp32 path.
constexpr int Q8_PLANE_SH_MAX = 126;

// Planes of one activation row held as float4 chunks, chunk c = tid + u*nth for u < NU
// (elements 4c..4c+3, block c/8).  nth must be a multiple of 32 so a block's 8 chunks sit
// in 8 consecutive lanes of one warp.  Writes planes[p*pstride + byte] (p = 0, 1, 2; byte in
// the Q8_0 row layout) and inv[block] = 2^-sh.  Every thread of the warps calls it.
template <int NU>
__device__ __forceinline__ void q8_build_planes(const float4 (&v)[NU], int K, int nth, int tid, uint8_t* planes,
                                                int pstride, float* inv) {
    const int nq = K >> 2;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        const int c = tid + u * nth;
        if (c - (tid & 31) >= nq) break;  // warp-uniform: no chunk of this warp is left
        const bool valid = c < nq;
        const float4 x = valid ? v[u] : make_float4(0.f, 0.f, 0.f, 0.f);
        float am = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
        if (!valid) continue;
        // am < 2^(e-126) for a normal am with biased exponent e: 2^sh = 2^(148-e) keeps
        // |x| * 2^sh below 2^22.  Zero and subnormal blocks take the largest shift.
        const int e = (int)((__float_as_uint(am) >> 23) & 0xFFu);
        const int sh = min(148 - e, Q8_PLANE_SH_MAX);
        const float S = __uint_as_float((uint32_t)(127 + sh) << 23);
        const float xv[4] = {x.x, x.y, x.z, x.w};
        // X = round(x * 2^sh): the scaling is exact and |X| < 2^22, so adding 1.5 * 2^23 rounds
        // to the integer (ties to even, as __float2int_rn) in the float's low mantissa bits.
        // Signed digits: x0 = the low byte of X; x1 = byte 1 of X + 128 (the carry of a
        // negative x0); x2 = byte 2 of X + 32896 (both carries).
        uint32_t X[4], Y1[4], Y2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            X[i] = (uint32_t)(__float_as_int(fmaf(xv[i], S, 12582912.0f)) - 0x4B400000);
            Y1[i] = X[i] + 128u;
            Y2[i] = X[i] + 32896u;
        }
        const uint32_t d0 = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
        const uint32_t d1 = __byte_perm(__byte_perm(Y1[0], Y1[1], 0x0051), __byte_perm(Y1[2], Y1[3], 0x0051), 0x5410);
        const uint32_t d2 = __byte_perm(__byte_perm(Y2[0], Y2[1], 0x0062), __byte_perm(Y2[2], Y2[3], 0x0062), 0x5410);
        const int b = c >> 3;
        const int off = 34 * b + 2 + 4 * (c & 7);  // even: 16-bit stores
        uint16_t* q0 = reinterpret_cast<uint16_t*>(planes + off);
        uint16_t* q1 = reinterpret_cast<uint16_t*>(planes + pstride + off);
        uint16_t* q2 = reinterpret_cast<uint16_t*>(planes + 2 * pstride + off);
        q0[0] = (uint16_t)d0;
        q0[1] = (uint16_t)(d0 >> 16);
        q1[0] = (uint16_t)d1;
        q1[1] = (uint16_t)(d1 >> 16);
        q2[0] = (uint16_t)d2;
        q2[1] = (uint16_t)(d2 >> 16);
        if ((c & 7) == 0) {
            const int so = 34 * b;  // the block's scale bytes meet zeros
            *reinterpret_cast<uint16_t*>(planes + so) = 0;
            *reinterpret_cast<uint16_t*>(planes + pstride + so) = 0;
            *reinterpret_cast<uint16_t*>(planes + 2 * pstride + so) = 0;
            // a non-finite block maximum makes the block's contribution NaN
            inv[b] = e == 255 ? __uint_as_float(0x7FC00000u) : __uint_as_float((uint32_t)(127 - sh) << 23);
        }
    }
}

// Q4_0 variant of the planes (the integer path for Q4_0 rows): the digits of block b sit in
// natural element order, plane p at planes[p*pstride + 32*b + j] (pstride = K), so a quant
// word's low nibbles (elements 4i..4i+3 of the block) meet plane word i and its high nibbles
// (elements 16+4i..) plane word 4+i; sums[4*b + p] = the signed digit sum of block b in plane
// p, for the -8 offset of the nibbles; inv[b] = 2^-sh.  Same digits as q8_build_planes.
// SUM16 (the Q6_K path): the sums are taken over 16-element halves instead and stored as
// 16-bit fields, word 4*b + p = (first half) | (second half) << 16 (|sum| <= 16 * 128).
template <int NU, bool SUM16 = false>
__device__ __forceinline__ void q4_build_planes(const float4 (&v)[NU], int K, int nth, int tid, uint8_t* planes,
                                                int pstride, float* inv, int* sums) {
    const int nq = K >> 2;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        const int c = tid + u * nth;
        if (c - (tid & 31) >= nq) break;  // warp-uniform: no chunk of this warp is left
        const bool valid = c < nq;
        const float4 x = valid ? v[u] : make_float4(0.f, 0.f, 0.f, 0.f);
        float am = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
        const int e = (int)((__float_as_uint(am) >> 23) & 0xFFu);
        const int sh = min(148 - e, Q8_PLANE_SH_MAX);
        const float S = __uint_as_float((uint32_t)(127 + sh) << 23);
        const float xv[4] = {x.x, x.y, x.z, x.w};
        uint32_t X[4], Y1[4], Y2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            X[i] = (uint32_t)(__float_as_int(fmaf(xv[i], S, 12582912.0f)) - 0x4B400000);
            Y1[i] = X[i] + 128u;
            Y2[i] = X[i] + 32896u;
        }
        const uint32_t d0 = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
        const uint32_t d1 = __byte_perm(__byte_perm(Y1[0], Y1[1], 0x0051), __byte_perm(Y1[2], Y1[3], 0x0051), 0x5410);
        const uint32_t d2 = __byte_perm(__byte_perm(Y2[0], Y2[1], 0x0062), __byte_perm(Y2[2], Y2[3], 0x0062), 0x5410);
        // digit sums per plane over the block's 8 lanes (SUM16: over each group of 4 lanes)
        int s0 = valid ? __dp4a((int)d0, 0x01010101, 0) : 0;
        int s1 = valid ? __dp4a((int)d1, 0x01010101, 0) : 0;
        int s2 = valid ? __dp4a((int)d2, 0x01010101, 0) : 0;
#pragma unroll
        for (int o = 1; o < (SUM16 ? 4 : 8); o <<= 1) {
            s0 += __shfl_xor_sync(0xffffffffu, s0, o);
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        if (!valid) continue;
        const int b = c >> 3;
        const int off = 32 * b + 4 * (c & 7);
        *reinterpret_cast<uint32_t*>(planes + off) = d0;
        *reinterpret_cast<uint32_t*>(planes + pstride + off) = d1;
        *reinterpret_cast<uint32_t*>(planes + 2 * pstride + off) = d2;
        if constexpr (SUM16) {
            if ((c & 3) == 0) {
                int16_t* h16 = reinterpret_cast<int16_t*>(sums + 4 * b) + ((c >> 2) & 1);
                h16[0] = (int16_t)s0;
                h16[2] = (int16_t)s1;
                h16[4] = (int16_t)s2;
            }
        } else if ((c & 7) == 0) {
            sums[4 * b] = s0;
            sums[4 * b + 1] = s1;
            sums[4 * b + 2] = s2;
        }
        if ((c & 7) == 0)
            inv[b] = e == 255 ? __uint_as_float(0x7FC00000u) : __uint_as_float((uint32_t)(127 - sh) << 23);
    }
}

// Bytes of one row's planes in memory: three planes of pstride bytes (the Q8_0 row layout,
// rounded up to 16 bytes) followed by the blocks' 2^-sh as floats.
__host__ __device__ constexpr int q8_plane_stride(int K) { return ((K / 32) * 34 + 15) & ~15; }
__host__ __device__ constexpr int q8_plane_bytes(int K) { return 3 * q8_plane_stride(K) + 4 * (K / 32); }

// Planes of one 32-element block b held one element per lane of a full warp: the same digits
// and 2^-sh as q8_build_planes, stored byte-wise at planes (any memory space).
__device__ __forceinline__ void q8_block_planes_warp(float x, int b, uint8_t* planes, int pstride, float* inv) {
    const int lane = threadIdx.x & 31;
    float am = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int e = (int)((__float_as_uint(am) >> 23) & 0xFFu);
    const int sh = min(148 - e, Q8_PLANE_SH_MAX);
    const float S = __uint_as_float((uint32_t)(127 + sh) << 23);
    const uint32_t X = (uint32_t)(__float_as_int(fmaf(x, S, 12582912.0f)) - 0x4B400000);
    uint8_t* q = planes + 34 * b + 2 + lane;
    q[0] = (uint8_t)X;
    q[pstride] = (uint8_t)((X + 128u) >> 8);
    q[2 * pstride] = (uint8_t)((X + 32896u) >> 16);
    if (lane < 6) planes[(lane >> 1) * pstride + 34 * b + (lane & 1)] = 0;  // the scale bytes
    if (lane == 0) inv[b] = e == 255 ? __uint_as_float(0x7FC00000u) : __uint_as_float((uint32_t)(127 - sh) << 23);
}

// One 64-element unit (two blocks, 17 words at wp) of one row against the lane's planes
// (the same unit's 17 words of each plane) and the two blocks' 2^-sh.
__device__ __forceinline__ float unit_dot_q8_int(const uint32_t* wp, const uint32_t (&pl)[51], float invA,
                                                 float invB) {
    int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
    uint32_t w0 = 0, w8 = 0;
#pragma unroll
    for (int i = 0; i < 9; ++i) {  // word 8 holds q30, q31 of block A and block B's scale
        const uint32_t w = wp[i];
        if (i == 0) w0 = w;
        if (i == 8) w8 = w;
        a0 = __dp4a((int)w, (int)pl[i], a0);
        a1 = __dp4a((int)w, (int)pl[17 + i], a1);
        a2 = __dp4a((int)w, (int)pl[34 + i], a2);
    }
#pragma unroll
    for (int i = 9; i < 17; ++i) {
        const uint32_t w = wp[i];
        b0 = __dp4a((int)w, (int)pl[i], b0);
        b1 = __dp4a((int)w, (int)pl[17 + i], b1);
        b2 = __dp4a((int)w, (int)pl[34 + i], b2);
    }
    const float dA = h2f(w0);
    const float dB = h2f(w8 >> 16);
    const float tA = fmaf((float)a2, 65536.f, (float)(a1 * 256 + a0));
    const float tB = fmaf((float)b2, 65536.f, (float)(b1 * 256 + b0));
    return fmaf(dA * invA, tA, (dB * invB) * tB);
}

// One 64-element unit of a Q4_0 row (two 18-byte blocks, 9 words at wp) against the lane's
// Q4_0 planes: pl[16p .. 16p+16) plane p's words of the two blocks, pl[48 + p] the two blocks'
// digit sums of plane p (block A in the low, block B in the high 16 bits).  Nibbles 0..15 are
// valid signed bytes for dp4a; the reference's q - 8 (src/quant.cpp:323-363) enters as
// -8 * (digit sum) per plane, so each plane's block sum stays an exact integer.
__device__ __forceinline__ float unit_dot_q4_int(const uint32_t* wp, const uint32_t (&pl)[51], float invA,
                                                 float invB) {
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = wp[i];
    int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t qa = __byte_perm(w[i], w[i + 1], 0x5432);  // block A's quant bytes 4i..4i+3
        const int la = (int)(qa & 0x0F0F0F0Fu), ha = (int)((qa >> 4) & 0x0F0F0F0Fu);
        a0 = __dp4a(la, (int)pl[i], a0);
        a0 = __dp4a(ha, (int)pl[4 + i], a0);
        a1 = __dp4a(la, (int)pl[16 + i], a1);
        a1 = __dp4a(ha, (int)pl[20 + i], a1);
        a2 = __dp4a(la, (int)pl[32 + i], a2);
        a2 = __dp4a(ha, (int)pl[36 + i], a2);
        const uint32_t qb = w[5 + i];  // block B's quant bytes
        const int lb = (int)(qb & 0x0F0F0F0Fu), hb = (int)((qb >> 4) & 0x0F0F0F0Fu);
        b0 = __dp4a(lb, (int)pl[8 + i], b0);
        b0 = __dp4a(hb, (int)pl[12 + i], b0);
        b1 = __dp4a(lb, (int)pl[24 + i], b1);
        b1 = __dp4a(hb, (int)pl[28 + i], b1);
        b2 = __dp4a(lb, (int)pl[40 + i], b2);
        b2 = __dp4a(hb, (int)pl[44 + i], b2);
    }
    a0 -= 8 * (int)(short)(pl[48] & 0xFFFFu);
    a1 -= 8 * (int)(short)(pl[49] & 0xFFFFu);
    a2 -= 8 * (int)(short)(pl[50] & 0xFFFFu);
    b0 -= 8 * ((int)pl[48] >> 16);
    b1 -= 8 * ((int)pl[49] >> 16);
    b2 -= 8 * ((int)pl[50] >> 16);
    const float dA = h2f(w[0]);
    const float dB = h2f(w[4] >> 16);
    const float tA = fmaf((float)a2, 65536.f, (float)(a1 * 256 + a0));
    const float tB = fmaf((float)b2, 65536.f, (float)(b1 * 256 + b0));
    return fmaf(dA * invA, tA, (dB * invB) * tB);
}

// One 64-element unit of a Q6_K row against the lane's natural-order planes (the Q4_0
// layout).  Unit (h, j) of a 256-element super-block (h = half, j = 0 / 1) holds the groups
// tq = j and tq = j + 2 of dequant_q6_K_row (src/quant.cpp:101-127): both read the 32 ql bytes
// at 64h + 32j (low / high nibbles) and the 32 qh bytes at 128 + 32h (bit pairs 2j / 2j + 4),
// so the unit is elements 128h + 32j + [0, 32) (activation block A) and 128h + 32(j + 2) +
// [0, 32) (block B = A + 2).  The six-bit u = ql nibble | qh bits << 4 (0..63) is a valid
// signed byte for dp4a; q = u - 32 enters as -32 * (the 16-element digit sums) per plane, so
// every 16-element sub-block sum stays an exact integer, which its int8 scale and the fp16 d
// then multiply.
//   sb:  the super-block (2-byte aligned: 210-byte blocks); sel: 0x3210 when sb is 4-byte
//        aligned, 0x5432 when it sits 2 bytes past a word (the words are realigned by PRMT)
//   pl:  pl[16p + i] plane p's words of block A (i < 8) and B (8 <= i < 16)
//   ss:  the SUM16 digit sums of block A (words 0..2: plane p, first half in the low and second
//        half in the high 16 bits) and of block B (words 8..10), in shared memory
__device__ __forceinline__ float unit_dot_q6k_int(const uint8_t* sb, int h, int j, uint32_t sel,
                                                  const uint32_t (&pl)[48], const uint32_t* ss, float invA,
                                                  float invB) {
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(sb) & ~(uintptr_t)3);
    const int qlw0 = (64 * h + 32 * j) >> 2, qhw0 = (128 + 32 * h) >> 2;
    const uint16_t* hw = reinterpret_cast<const uint16_t*>(sb);  // sb is 2-byte aligned
    const uint32_t scA = hw[96 + 4 * h + j];                     // scales[8h + 2j], [8h + 2j + 1]
    const uint32_t scB = hw[96 + 4 * h + j + 2];                 // scales[8h + 2j + 4], [.. + 5]
    const float d = h2f(hw[104]);
    const int shA = 4 - 2 * j, shB = 2 * j;
    float fA = 0.f, fB = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
        uint32_t ql[5], qh[5];  // this half's words (one more for the realignment)
#pragma unroll
        for (int k = 0; k < 5; ++k) {
            ql[k] = aw[qlw0 + 4 * half + k];
            qh[k] = aw[qhw0 + 4 * half + k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = 4 * half + k;
            const uint32_t lw = __byte_perm(ql[k], ql[k + 1], sel);
            const uint32_t hq = __byte_perm(qh[k], qh[k + 1], sel);
            const int uA = (int)((lw & 0x0F0F0F0Fu) | ((hq << shA) & 0x30303030u));
            const int uB = (int)(((lw >> 4) & 0x0F0F0F0Fu) | ((hq >> shB) & 0x30303030u));
            a0 = __dp4a(uA, (int)pl[i], a0);
            a1 = __dp4a(uA, (int)pl[16 + i], a1);
            a2 = __dp4a(uA, (int)pl[32 + i], a2);
            b0 = __dp4a(uB, (int)pl[8 + i], b0);
            b1 = __dp4a(uB, (int)pl[24 + i], b1);
            b2 = __dp4a(uB, (int)pl[40 + i], b2);
        }
        // 16-element digit sums of this half (signed 16-bit fields)
        const int sh16 = half ? 0 : 16;
        const uint4 sa = *reinterpret_cast<const uint4*>(ss), sbb = *reinterpret_cast<const uint4*>(ss + 8);
        a0 -= 32 * ((int)(sa.x << sh16) >> 16);
        a1 -= 32 * ((int)(sa.y << sh16) >> 16);
        a2 -= 32 * ((int)(sa.z << sh16) >> 16);
        b0 -= 32 * ((int)(sbb.x << sh16) >> 16);
        b1 -= 32 * ((int)(sbb.y << sh16) >> 16);
        b2 -= 32 * ((int)(sbb.z << sh16) >> 16);
        const float tA = fmaf((float)a2, 65536.f, (float)(a1 * 256 + a0));
        const float tB = fmaf((float)b2, 65536.f, (float)(b1 * 256 + b0));
        const float sA = (float)(int8_t)(scA >> (8 * half)), sB = (float)(int8_t)(scB >> (8 * half));
        fA = fmaf(sA, tA, fA);
        fB = fmaf(sB, tB, fB);
    }
    return d * fmaf(invA, fA, invB * fB);
}

// ---- Q8_0 fast path: one row segment of `units` 64-element units -----------------------
// Products and partial sums use the packed fp32x2 pipe of sm_100 (__ffma2_rn / __fadd2_rn):
// two weights per instruction, each lane still forming exact fp32 x*q products.
template <int MAXM>
__device__ __forceinline__ void dot_q8_fast(const uint8_t* seg, int units, const float* xseg, int xl, int M,
                                            int lane, float (&acc)[MAXM]) {
    const float2 kBias = make_float2(-8388736.0f, -8388736.0f);
    for (int u = lane; u < units; u += 32) {
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(seg + (size_t)u * 68);
        uint32_t w[17];
#pragma unroll
        for (int i = 0; i < 17; ++i) w[i] = wp[i];
        const float dA = h2f(w[0]);
        const float dB = h2f(w[8] >> 16);
#pragma unroll
        for (int i = 0; i < 17; ++i) w[i] ^= 0x80808080u;
        const float* xu = xseg + (size_t)u * 68;
        float2 sA[MAXM][2], sB[MAXM][2];
#pragma unroll
        for (int m = 0; m < MAXM; ++m)
#pragma unroll
            for (int r = 0; r < 2; ++r) sA[m][r] = sB[m][r] = make_float2(0.f, 0.f);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            float qa[4], qb[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int ja = 2 + 4 * g + e;  // byte of block A within the unit
                const int jb = 36 + 4 * g + e; // byte of block B
                qa[e] = __int_as_float((int)__byte_perm(w[ja >> 2], 0x4B000000u, 0x7650u | (uint32_t)(ja & 3)));
                qb[e] = __int_as_float((int)__byte_perm(w[jb >> 2], 0x4B000000u, 0x7650u | (uint32_t)(jb & 3)));
            }
            const float2 qa0 = __fadd2_rn(make_float2(qa[0], qa[1]), kBias);
            const float2 qa1 = __fadd2_rn(make_float2(qa[2], qa[3]), kBias);
            const float2 qb0 = __fadd2_rn(make_float2(qb[0], qb[1]), kBias);
            const float2 qb1 = __fadd2_rn(make_float2(qb[2], qb[3]), kBias);
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M) {
                    const float4 xa = *reinterpret_cast<const float4*>(xu + m * xl + 4 * g);
                    const float4 xb = *reinterpret_cast<const float4*>(xu + m * xl + 32 + 4 * g);
                    float2& a2 = sA[m][g & 1];
                    float2& b2 = sB[m][g & 1];
                    a2 = __ffma2_rn(make_float2(xa.x, xa.y), qa0, a2);
                    a2 = __ffma2_rn(make_float2(xa.z, xa.w), qa1, a2);
                    b2 = __ffma2_rn(make_float2(xb.x, xb.y), qb0, b2);
                    b2 = __ffma2_rn(make_float2(xb.z, xb.w), qb1, b2);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            const float2 a2 = __fadd2_rn(sA[m][0], sA[m][1]);
            const float2 b2 = __fadd2_rn(sB[m][0], sB[m][1]);
            acc[m] = fmaf(dA, a2.x + a2.y, acc[m]);
            acc[m] = fmaf(dB, b2.x + b2.y, acc[m]);
        }
    }
}

// ---- generic path: one lane per 32-element group of a block -------------------------------
// Produces either (scale, q[32]) with the block scale applied to the block sum (Q8_0, Q4_0,
// as src/quant.cpp:266-363 do) or dequantised w[32] (Q4_1, Q6_K, F16, F32, as
// dequant_row + dot_f32 do).  A Q6_K super-block's eight groups go to eight lanes, so a
// 2048-element row keeps every lane of the warp busy.
template <int MAXM>
__device__ __forceinline__ void dot_generic(int t, const uint8_t* seg, int e0, int nelem, const float* xs, int xl,
                                            int M, int lane, float (&acc)[MAXM]) {
    const int be = (t == T_Q6_K) ? 256 : 32;
    const int bb = (t == T_F32) ? 128 : (t == T_F16) ? 64 : blk_bytes(t);
    const int groups = be / 32;
    const int nwork = (nelem / be) * groups;
    for (int wi = lane; wi < nwork; wi += 32) {
        const int b = groups == 1 ? wi : wi >> 3, g = groups == 1 ? 0 : wi & 7;
        const uint8_t* p = seg + (size_t)b * bb;
        {
            float w[32];
            float scale = 1.f;
            bool scaled = false;
            if (t == T_Q8_0) {
                scale = h2f(ld_u16(p));
                scaled = true;
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = (float)(int8_t)p[2 + j];
            } else if (t == T_Q4_0) {
                scale = h2f(ld_u16(p));
                scaled = true;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const uint32_t q = p[2 + j];
                    w[j] = (float)((int)(q & 15u) - 8);
                    w[j + 16] = (float)((int)(q >> 4) - 8);
                }
            } else if (t == T_Q4_1) {
                const float d = h2f(ld_u16(p)), mn = h2f(ld_u16(p + 2));
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const uint32_t q = p[4 + j];
                    w[j] = __fmaf_rn((float)(q & 15u), d, mn);
                    w[j + 16] = __fmaf_rn((float)(q >> 4), d, mn);
                }
            } else if (t == T_Q6_K) {
                const int h = g >> 2, tq = g & 3;
                const float d = h2f(ld_u16(p + 208));
                const uint8_t* ql = p + 64 * h + ((tq & 1) ? 32 : 0);
                const uint8_t* qh = p + 128 + 32 * h;
                const int8_t* sc = reinterpret_cast<const int8_t*>(p + 192 + 8 * h + 2 * tq);
                const float ds0 = __fmul_rn(d, (float)sc[0]);
                const float ds1 = __fmul_rn(d, (float)sc[1]);
#pragma unroll
                for (int l = 0; l < 32; ++l) {
                    const uint32_t lo = (tq >= 2) ? (ql[l] >> 4) : (ql[l] & 15u);
                    const uint32_t hi = (qh[l] >> (2 * tq)) & 3u;
                    const int q = (int)(lo | (hi << 4)) - 32;
                    w[l] = __fmul_rn(l < 16 ? ds0 : ds1, (float)q);
                }
            } else if (t == T_F16) {
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = h2f(ld_u16(p + 2 * j));
            } else {  // F32: rows are 4-byte aligned
                const float* fp = reinterpret_cast<const float*>(p);
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = fp[j];
            }
            const int ebase = e0 + b * be + 32 * g;
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M) {
                    const float* xm = xs + m * xl;
                    float s = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) s = fmaf(xm[xpad(ebase + j)], w[j], s);
                    acc[m] = scaled ? fmaf(scale, s, acc[m]) : acc[m] + s;
                }
            }
        }
    }
}

// ---- embedding row dequantisation into shared memory (dequant_row, src/quant.cpp:133) ---
static __device__ void embed_row(float* xm, const uint8_t* E, int t, long long rb, int K, long long tok, int nthreads) {
    const uint8_t* row = E + tok * rb;
    const int be = (t == T_Q6_K) ? 256 : 32;
    const int bb = (t == T_F32) ? 128 : (t == T_F16) ? 64 : blk_bytes(t);
    const int tid = threadIdx.x;
    const int nb = K / be;
    for (int b = tid; b < nb; b += nthreads) {
        const uint8_t* p = row + (size_t)b * bb;
        for (int g = 0; g < be / 32; ++g) {
            const int e = b * be + 32 * g;
            for (int j = 0; j < 32; ++j) {
                float v;
                if (t == T_Q8_0) {
                    v = __fmul_rn(h2f(ld_u16(p)), (float)(int8_t)p[2 + j]);
                } else if (t == T_Q4_0) {
                    const uint32_t q = p[2 + (j & 15)];
                    v = __fmul_rn(h2f(ld_u16(p)), (float)((int)((j < 16) ? (q & 15u) : (q >> 4)) - 8));
                } else if (t == T_Q4_1) {
                    const uint32_t q = p[4 + (j & 15)];
                    v = __fmaf_rn((float)((j < 16) ? (q & 15u) : (q >> 4)), h2f(ld_u16(p)), h2f(ld_u16(p + 2)));
                } else if (t == T_Q6_K) {
                    const int h = g >> 2, tq = g & 3;
                    const uint8_t* ql = p + 64 * h + ((tq & 1) ? 32 : 0);
                    const uint8_t* qh = p + 128 + 32 * h;
                    const int8_t sc = reinterpret_cast<const int8_t*>(p + 192 + 8 * h + 2 * tq)[j >> 4];
                    const uint32_t lo = (tq >= 2) ? (ql[j] >> 4) : (ql[j] & 15u);
                    const uint32_t hi = (qh[j] >> (2 * tq)) & 3u;
                    v = __fmul_rn(__fmul_rn(h2f(ld_u16(p + 208)), (float)sc), (float)((int)(lo | (hi << 4)) - 32));
                } else if (t == T_F16) {
                    v = h2f(ld_u16(p + 2 * (32 * g + j)));
                } else {
                    v = reinterpret_cast<const float*>(p)[32 * g + j];
                }
                xm[xpad(e + j)] = v;
            }
        }
    }
}

}  // namespace tfb
