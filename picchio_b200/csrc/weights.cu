// weights.cu - weight preparation on the device: re-tiling of INT4/INT8
// matrices from the reference's host layout (quant.h:32-41) into the GEMV
// tile layout (layout.h), the inverse dequant view used by the tests, and
// seeded synthetic weights quantized as the reference converter does
// (convert.py:45-126).
#include <cuda_bf16.h>

#include <cstdint>

#include "kernels.h"

namespace pc {

namespace {

__device__ __forceinline__ int src_nibble(const uint8_t *q4, int O, int I, int row, int col, int pad) {
    if (row >= O || col >= I) return pad;  // padding: value 0
    const uint8_t b = q4[(int64_t)row * ((I + 1) / 2) + (col >> 1)];
    return (col & 1) ? (b >> 4) : (b & 0xF);
}

// One thread per (row tile, block, lane): 16 bytes of nibbles (+ the scales
// of rows g and g+8 for lanes with t == 0).  Word q = 2m + h of lane 4g + t
// holds columns 64kc + 32m + 16h + 4t + j (j = 0..3): for INT4 in byte j, row
// g in the low nibble and row g + 8 in the high nibble; for MXFP4 (F4) row
// g's codes in bits 4j..4j+3 and row g + 8's in bits 16 + 4j.. (the source
// layout is the same for both: two 4-bit values per byte, low nibble = even
// column, as quant.h:32-41 and the MXFP4 blocks of convert.py:413-420 store
// them).  Padding is the value 0: nibble 8 for INT4, code 0 for MXFP4.
__global__ void retile_t4_kernel(const uint8_t *q4, const float *scales, int bs, TileDesc d) {
    const bool f4 = d.fmt == TF_F4;
    const int64_t total = (int64_t)(d.Op / 16) * d.kblocks * 32;
    const int ng = bs > 0 ? (d.I + bs - 1) / bs : 1;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int L = (int)(idx & 31);
        const int64_t blk = idx >> 5;
        const int kc = (int)(blk % d.kblocks), rt = (int)(blk / d.kblocks);
        const int g = L >> 2, t = L & 3;
        const int rlo = tile_row_to_logical(d.perm, d.head_dim, rt, g);
        const int rhi = tile_row_to_logical(d.perm, d.head_dim, rt, g + 8);
        uint32_t w[4];
        for (int q = 0; q < 4; ++q) {
            const int c = kc * 64 + 32 * (q >> 1) + 16 * (q & 1) + 4 * t;
            uint32_t v = 0;
            for (int j = 0; j < 4; ++j) {
                const uint32_t lo = src_nibble(q4, d.O, d.I, rlo, c + j, f4 ? 0 : 8);
                const uint32_t hi = src_nibble(q4, d.O, d.I, rhi, c + j, f4 ? 0 : 8);
                v |= f4 ? (lo << (4 * j)) | (hi << (16 + 4 * j)) : (lo << (8 * j)) | (hi << (8 * j + 4));
            }
            w[q] = v;
        }
        uint8_t *dst = d.tiles + blk * d.blk_bytes;
        *reinterpret_cast<uint4 *>(dst + L * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        if (d.gs > 0 && t == 0) {
            const int gpc = 64 / d.gs;
            float *sd = reinterpret_cast<float *>(dst + 512);
            for (int j = 0; j < gpc; ++j) {
                const int gi = kc * gpc + j;
                const bool in = gi * d.gs < d.I;
                sd[g * gpc * 2 + j * 2 + 0] = (rlo < d.O && in) ? scales[(int64_t)rlo * ng + gi] : 0.0f;
                sd[g * gpc * 2 + j * 2 + 1] = (rhi < d.O && in) ? scales[(int64_t)rhi * ng + gi] : 0.0f;
            }
        }
    }
}

__device__ __forceinline__ uint32_t src_byte(const int8_t *q8, int O, int I, int row, int col) {
    if (row >= O || col >= I) return 0u;
    return (uint32_t)(uint8_t)q8[(int64_t)row * I + col];
}

// Word 2h + r of lane 4g + t holds columns 32kc + 16h + 4t + j in byte j, of
// row g (r = 0) or g + 8 (r = 1): the lane's A fragment of one m16n8k32 step.
__global__ void retile_t8_kernel(const int8_t *q8, TileDesc d) {
    const int64_t total = (int64_t)(d.Op / 16) * d.kblocks * 32;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int L = (int)(idx & 31);
        const int64_t blk = idx >> 5;
        const int kc = (int)(blk % d.kblocks), rt = (int)(blk / d.kblocks);
        const int g = L >> 2, t = L & 3;
        const int rows[2] = {tile_row_to_logical(d.perm, d.head_dim, rt, g),
                             tile_row_to_logical(d.perm, d.head_dim, rt, g + 8)};
        uint32_t w[4];
        for (int q = 0; q < 4; ++q) {
            const int c = kc * 32 + 16 * (q >> 1) + 4 * t, r = rows[q & 1];
            w[q] = src_byte(q8, d.O, d.I, r, c) | (src_byte(q8, d.O, d.I, r, c + 1) << 8) |
                   (src_byte(q8, d.O, d.I, r, c + 2) << 16) | (src_byte(q8, d.O, d.I, r, c + 3) << 24);
        }
        *reinterpret_cast<uint4 *>(d.tiles + blk * d.blk_bytes + L * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void copy_rs_kernel(const float *scales, float *rs, int O, int Op) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Op; i += gridDim.x * blockDim.x)
        rs[i] = i < O ? scales[i] : 0.0f;
}

// logical row -> (row tile, tile row)
__device__ __forceinline__ void logical_to_tile(int perm, int hd, int lr, int &rt, int &tr) {
    if (perm == PERM_PAIR) {
        const int p = lr >> 1;
        rt = p >> 3;
        tr = (p & 7) + 8 * (lr & 1);
    } else if (perm == PERM_HEAD) {
        const int half = hd / 2, h = lr / hd, jj = lr % hd, hi = jj >= half, j = jj - hi * half;
        rt = h * (hd / 16) + j / 8;
        tr = (j & 7) + 8 * hi;
    } else {
        rt = lr >> 4;
        tr = lr & 15;
    }
}

__global__ void dequant_tiles_kernel(TileDesc d, float *out) {
    const int64_t total = (int64_t)d.O * d.I;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int lr = (int)(idx / d.I), c = (int)(idx % d.I);
        int rt, tr;
        logical_to_tile(d.perm, d.head_dim, lr, rt, tr);
        const int g = tr & 7, rh = tr >> 3;
        float v, s;
        if (tf_4bit(d.fmt)) {
            const int kc = c / 64, r = c % 64;
            const int q = 2 * (r / 32) + (r % 32) / 16, t = (r % 16) / 4, j = r % 4;
            const uint8_t *blk = d.tiles + ((int64_t)rt * d.kblocks + kc) * d.blk_bytes;
            const uint32_t w = *reinterpret_cast<const uint32_t *>(blk + (4 * g + t) * 16 + q * 4);
            if (d.fmt == TF_F4) {  // E2M1 (convert.py:98-103): code 8 is -0
                const int code = (int)((w >> (4 * j + 16 * rh)) & 0xF);
                const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
                v = (code & 8) ? -mag[code & 7] : mag[code & 7];
            } else {
                v = (float)((int)((w >> (8 * j + 4 * rh)) & 0xF) - 8);
            }
            if (d.gs > 0) {
                const int gpc = 64 / d.gs, jg = r / d.gs;
                s = reinterpret_cast<const float *>(blk + 512)[g * gpc * 2 + jg * 2 + rh];
            } else {
                s = d.rs[lr];
            }
        } else {
            const int kc = c / 32, r = c % 32;
            const int q = 2 * (r / 16) + rh, t = (r % 16) / 4, j = r % 4;
            const uint8_t *blk = d.tiles + ((int64_t)rt * d.kblocks + kc) * d.blk_bytes;
            const uint32_t w = *reinterpret_cast<const uint32_t *>(blk + (4 * g + t) * 16 + q * 4);
            v = (float)(int8_t)((w >> (8 * j)) & 0xFF);
            s = d.rs[lr];
        }
        out[idx] = __fmul_rn(v, s);
    }
}

// ---- seeded normals: splitmix64 counter hash + Box-Muller ----
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
    const uint64_t r = mix64(seed ^ mix64(i));
    const float u1 = ((float)(uint32_t)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = (float)(uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void gen_i4_kernel(uint8_t *q4, float *scales, int O, int I, int gs, uint64_t seed, float sd) {
    const int ng = gs > 0 ? (I + gs - 1) / gs : 1;
    const int64_t total = (int64_t)O * ng;
    const int rb = (I + 1) / 2;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(idx / ng), g = (int)(idx % ng);
        const int c0 = gs > 0 ? g * gs : 0, c1 = gs > 0 ? min(c0 + gs, I) : I;
        float amax = 0.0f;
        for (int c = c0; c < c1; ++c)
            amax = fmaxf(amax, fabsf(__fmul_rn(normal_at(seed, (uint64_t)row * I + c), sd)));
        const float s = amax > 1e-8f ? __fdiv_rn(amax, 7.0f) : 1e-8f;
        scales[idx] = s;
        for (int c = c0; c < c1; c += 2) {
            int v0 = (int)rintf(__fdiv_rn(__fmul_rn(normal_at(seed, (uint64_t)row * I + c), sd), s));
            v0 = max(-8, min(7, v0));
            int v1 = 0;
            if (c + 1 < c1) {
                v1 = (int)rintf(__fdiv_rn(__fmul_rn(normal_at(seed, (uint64_t)row * I + c + 1), sd), s));
                v1 = max(-8, min(7, v1));
            }
            q4[(int64_t)row * rb + (c >> 1)] = (uint8_t)((v0 + 8) | ((v1 + 8) << 4));
        }
    }
}

// MXFP4 per the OCP microscaling rule, one thread per 32-column block: the
// shared exponent is floor(log2(max |w|)) - 2 (2 = the largest E2M1
// exponent), clamped to [-127, 127], stored as the E8M0 byte + 127; each
// w / 2^exp rounds to the nearest E2M1 value (0, 0.5, 1, 1.5, 2, 3, 4, 6;
// ties to the even code; beyond 6 saturates), sign in bit 3.  The decoded
// scale 2^exp goes to `scales` as a float.
__device__ __forceinline__ int e2m1_code(float v) {
    const float a = fabsf(v);
    const float mids[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
    int idx = 0;
    for (int i = 0; i < 7; ++i) idx += mids[i] < a;
    if (idx < 7 && a == mids[idx] && (idx & 1)) ++idx;  // tie: the even code
    return idx | (v < 0.0f ? 8 : 0);
}

__global__ void gen_f4_kernel(uint8_t *q4, float *scales, int O, int I, uint64_t seed, float sd) {
    const int nb = I / 32;
    const int64_t total = (int64_t)O * nb;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(idx / nb), b = (int)(idx % nb);
        float w[32], amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            w[j] = __fmul_rn(normal_at(seed, (uint64_t)row * I + b * 32 + j), sd);
            amax = fmaxf(amax, fabsf(w[j]));
        }
        int ex = amax > 0.0f ? (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 2 : -127;
        ex = max(-127, min(127, ex));
        const float inv = ldexpf(1.0f, -ex), sc = ldexpf(1.0f, ex);
        scales[idx] = sc;
        for (int j = 0; j < 32; j += 2) {
            const int c0 = e2m1_code(__fmul_rn(w[j], inv)), c1 = e2m1_code(__fmul_rn(w[j + 1], inv));
            q4[(int64_t)row * (I / 2) + b * 16 + j / 2] = (uint8_t)(c0 | (c1 << 4));
        }
    }
}

__global__ void gen_i8_kernel(int8_t *q8, float *scales, int O, int I, uint64_t seed, float sd) {
    for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < O; row += gridDim.x * blockDim.x) {
        float amax = 0.0f;
        for (int c = 0; c < I; ++c)
            amax = fmaxf(amax, fabsf(__fmul_rn(normal_at(seed, (uint64_t)row * I + c), sd)));
        const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
        scales[row] = s;
        for (int c = 0; c < I; ++c) {
            int v = (int)rintf(__fdiv_rn(__fmul_rn(normal_at(seed, (uint64_t)row * I + c), sd), s));
            q8[(int64_t)row * I + c] = (int8_t)max(-127, min(127, v));
        }
    }
}

__global__ void gen_f32_kernel(float *dst, int64_t n, uint64_t seed, float mean, float sd) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __fadd_rn(mean, __fmul_rn(sd, normal_at(seed, (uint64_t)i)));
}

__global__ void gen_kv_kernel(void *base, int64_t off, int64_t n, int bf16, uint64_t seed) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = normal_at(seed, (uint64_t)i);
        if (bf16)
            reinterpret_cast<__nv_bfloat16 *>(base)[off + i] = __float2bfloat16_rn(v);
        else
            reinterpret_cast<float *>(base)[off + i] = v;
    }
}

int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    return (int)(b < 1 ? 1 : (b > 148 * 64 ? 148 * 64 : b));
}

}  // namespace

cudaError_t retile_t4(const uint8_t *q4, const float *scales, int src_block_size, TileDesc &d, cudaStream_t st) {
    const int64_t total = (int64_t)(d.Op / 16) * d.kblocks * 32;
    retile_t4_kernel<<<grid_for(total, 256), 256, 0, st>>>(q4, scales, src_block_size, d);
    if (d.gs == 0) copy_rs_kernel<<<grid_for(d.Op, 256), 256, 0, st>>>(scales, d.rs, d.O, d.Op);
    return cudaGetLastError();
}

cudaError_t retile_t8(const int8_t *q8, const float *scales, TileDesc &d, cudaStream_t st) {
    const int64_t total = (int64_t)(d.Op / 16) * d.kblocks * 32;
    retile_t8_kernel<<<grid_for(total, 256), 256, 0, st>>>(q8, d);
    copy_rs_kernel<<<grid_for(d.Op, 256), 256, 0, st>>>(scales, d.rs, d.O, d.Op);
    return cudaGetLastError();
}

cudaError_t dequant_tiles(const TileDesc &d, float *out, cudaStream_t st) {
    dequant_tiles_kernel<<<grid_for((int64_t)d.O * d.I, 256), 256, 0, st>>>(d, out);
    return cudaGetLastError();
}

cudaError_t gen_i4_rowmajor(uint8_t *q4, float *scales, int O, int I, int gs, uint64_t seed, float sd,
                            cudaStream_t st) {
    const int ng = gs > 0 ? (I + gs - 1) / gs : 1;
    gen_i4_kernel<<<grid_for((int64_t)O * ng, 128), 128, 0, st>>>(q4, scales, O, I, gs, seed, sd);
    return cudaGetLastError();
}

cudaError_t gen_f4_rowmajor(uint8_t *q4, float *scales, int O, int I, uint64_t seed, float sd, cudaStream_t st) {
    if (I % 32) return cudaErrorInvalidValue;
    gen_f4_kernel<<<grid_for((int64_t)O * (I / 32), 128), 128, 0, st>>>(q4, scales, O, I, seed, sd);
    return cudaGetLastError();
}

cudaError_t gen_i8_rowmajor(int8_t *q8, float *scales, int O, int I, uint64_t seed, float sd, cudaStream_t st) {
    gen_i8_kernel<<<grid_for(O, 64), 64, 0, st>>>(q8, scales, O, I, seed, sd);
    return cudaGetLastError();
}

cudaError_t gen_kv(void *base, int64_t off, int64_t n, int bf16, uint64_t seed, cudaStream_t st) {
    gen_kv_kernel<<<grid_for(n, 256), 256, 0, st>>>(base, off, n, bf16, seed);
    return cudaGetLastError();
}

cudaError_t gen_f32(float *dst, int64_t n, uint64_t seed, float mean, float sd, cudaStream_t st) {
    gen_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, n, seed, mean, sd);
    return cudaGetLastError();
}

}  // namespace pc
