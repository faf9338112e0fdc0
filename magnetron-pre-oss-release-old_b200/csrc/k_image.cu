// Image tensors on the device: the pixel work of mag_tensor_load_image /
// mag_tensor_save_image (magnetron/magnetron.c:3013-3109) and of
// mag_tensor_img_draw_box / mag_tensor_img_draw_text (magnetron/magnetron.c:2159-2270).
//
// An image tensor is planar f32 [c][h][w] (shape (c, h, w), x fastest); decoded
// files are interleaved u8 [h][w][c].  Every f32 step follows the reference's
// operation order with separately rounded multiply and add (no contraction), so
// the results are bit-identical.
#include "mcu_glyphs.cuh"
#include "mcu_kernels.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kImgThreads = 256;

__device__ __forceinline__ float u8_unit(const uint8_t* __restrict__ src, uint32_t idx) {
    return __fdiv_rn((float)src[idx], 255.0f);
}

// Interleaved u8 -> planar f32 / 255 (magnetron/magnetron.c:3070-3077): one thread per pixel.
__global__ void __launch_bounds__(kImgThreads) img_from_u8(float* __restrict__ dst, const uint8_t* __restrict__ src,
                                                           uint32_t w, uint32_t h, uint32_t c) {
    const uint64_t px = (uint64_t)blockIdx.x * kImgThreads + threadIdx.x;
    const uint64_t plane = (uint64_t)w * h;
    if (px >= plane) return;
    for (uint32_t k = 0; k < c; ++k) dst[px + plane * k] = u8_unit(src, (uint32_t)(px * c + k));
}

// The horizontal pass of the reference resize (magnetron/magnetron.c:3030-3047) at
// output column cc of source row `row`, channel k.
__device__ __forceinline__ float resize_h(const uint8_t* __restrict__ src, uint32_t w, uint32_t c, uint32_t k,
                                          uint32_t row, uint32_t cc, uint32_t rw, float ws) {
    const uint32_t base = row * w;
    if (cc == rw - 1 || w == 1) return u8_unit(src, (base + (w - 1)) * c + k);
    const float sx = __fmul_rn((float)cc, ws);
    uint32_t ix = (uint32_t)sx;
    const float dx = __fsub_rn(sx, (float)ix);
    if (ix > w - 2) ix = w - 2;  // in range for every size the reference reads in range
    const float a = u8_unit(src, (base + ix) * c + k), b = u8_unit(src, (base + ix + 1) * c + k);
    return __fadd_rn(__fmul_rn(__fsub_rn(1.0f, dx), a), __fmul_rn(dx, b));
}

// Bilinear resize fused with the conversion: the vertical pass (magnetron/magnetron.c:3048-3062)
// over two horizontal-pass values per output pixel; one thread per output pixel and channel.
__global__ void __launch_bounds__(kImgThreads) img_from_u8_resized(float* __restrict__ dst,
                                                                   const uint8_t* __restrict__ src, uint32_t w,
                                                                   uint32_t h, uint32_t c, uint32_t rw, uint32_t rh,
                                                                   float ws, float hs) {
    const uint64_t i = (uint64_t)blockIdx.x * kImgThreads + threadIdx.x;
    const uint64_t plane = (uint64_t)rw * rh;
    if (i >= plane * c) return;
    const uint32_t k = (uint32_t)(i / plane);
    const uint32_t rem = (uint32_t)(i - (uint64_t)k * plane);
    const uint32_t r = rem / rw, cc = rem - r * rw;
    const float sy = __fmul_rn((float)r, hs);
    uint32_t iy = (uint32_t)sy;  // NaN (rh == 1) converts to 0, as on x86
    const float dy = __fsub_rn(sy, (float)iy);
    if (iy > h - 1) iy = h - 1;
    float v = __fmul_rn(__fsub_rn(1.0f, dy), resize_h(src, w, c, k, iy, cc, rw, ws));
    if (!(r == rh - 1 || h == 1)) {
        const uint32_t iy1 = iy + 1 < h ? iy + 1 : h - 1;
        v = __fadd_rn(v, __fmul_rn(dy, resize_h(src, w, c, k, iy1, cc, rw, ws)));
    }
    dst[i] = v;
}

// Planar f32 -> interleaved u8 as (uint8_t)(x * 255.0f) compiles on x86-64
// (magnetron/magnetron.c:3101-3103): truncation to int32 (0x80000000 when out of
// range or NaN), then the low byte.
__global__ void __launch_bounds__(kImgThreads) img_to_u8(uint8_t* __restrict__ dst, const float* __restrict__ src,
                                                         uint32_t w, uint32_t h, uint32_t c) {
    const uint64_t px = (uint64_t)blockIdx.x * kImgThreads + threadIdx.x;
    const uint64_t plane = (uint64_t)w * h;
    if (px >= plane) return;
    for (uint32_t k = 0; k < c; ++k) {
        const float v = __fmul_rn(src[px + plane * k], 255.0f);
        const int32_t q = (v >= -2147483648.0f && v < 2147483648.0f) ? (int32_t)v : INT32_MIN;
        dst[px * c + k] = (uint8_t)q;
    }
}

__device__ __forceinline__ void put_rgb(float* __restrict__ img, int64_t plane, int32_t w, int32_t x, int32_t y,
                                        float r, float g, float b) {
    const int64_t o = x + (int64_t)y * w;
    if (o < 0 || o >= plane) return;  // where the reference's bounds check fails
    img[o] = r;
    img[o + plane] = g;
    img[o + 2 * plane] = b;
}

// draw_box (magnetron/magnetron.c:2170-2212): ring i, clamped to the image, gets its two
// horizontal edges (x in [xx1, xx2]) and two vertical edges (y in [yy1, yy2]).  A column
// below zero lands on the previous row, as in the reference.
__global__ void __launch_bounds__(kImgThreads) img_draw_box(float* __restrict__ img, int32_t w, int32_t h,
                                                            int32_t x1, int32_t y1, int32_t x2, int32_t y2,
                                                            int32_t wi, float r, float g, float b) {
    const int64_t plane = (int64_t)w * h;
    const int32_t stride = gridDim.x * kImgThreads;
    for (int32_t i = blockIdx.y; i < wi; i += gridDim.y) {
        int32_t xx1 = x1 + i, yy1 = y1 + i, xx2 = x2 - i, yy2 = y2 - i;
        if (xx1 >= w) xx1 = w - 1;
        if (xx2 >= w) xx2 = w - 1;
        if (yy1 >= h) yy1 = h - 1;
        if (yy2 >= h) yy2 = h - 1;
        for (int32_t j = xx1 + (int32_t)(blockIdx.x * kImgThreads + threadIdx.x); j <= xx2; j += stride) {
            put_rgb(img, plane, w, j, yy1, r, g, b);
            put_rgb(img, plane, w, j, yy2, r, g, b);
        }
        for (int32_t j = yy1 + (int32_t)(blockIdx.x * kImgThreads + threadIdx.x); j <= yy2; j += stride) {
            put_rgb(img, plane, w, xx1, j, r, g, b);
            put_rgb(img, plane, w, xx2, j, r, g, b);
        }
    }
}

// draw_text: one CTA per placed glyph, one thread per cell of its 8 x 14 box.
__global__ void __launch_bounds__(128) img_draw_text(float* __restrict__ img, int32_t w, int32_t h,
                                                     const int32_t* __restrict__ glyphs, float r, float g, float b) {
    const int32_t* q = glyphs + 3 * blockIdx.x;  // x, y, glyph index 0..93
    const int32_t xx = threadIdx.x & 7, yy = threadIdx.x >> 3;
    if (yy >= 14 || xx == 0) return;  // column 0 of the box is never set
    if (!((mcu_glyph_rows[q[2] * 14 + yy] >> (xx - 1)) & 1)) return;
    const int32_t px = q[0] + xx, py = q[1] + yy;
    if (px >= w || py >= h) return;
    const int64_t plane = (int64_t)w * h, o = (int64_t)py * w + px;
    img[o] = r;
    img[o + plane] = g;
    img[o + 2 * plane] = b;
}

inline int blocks_for(uint64_t n) { return (int)((n + kImgThreads - 1) / kImgThreads); }

}  // namespace

extern "C" int mcu_launch_img_from_u8(float* dst, const uint8_t* src, uint32_t w, uint32_t h, uint32_t c, uint32_t rw,
                                      uint32_t rh, float ws, float hs, cudaStream_t st) {
    if (rw && rh) {
        const uint64_t n = (uint64_t)rw * rh * c;
        if (!n) return 0;
        img_from_u8_resized<<<blocks_for(n), kImgThreads, 0, st>>>(dst, src, w, h, c, rw, rh, ws, hs);
    } else {
        const uint64_t n = (uint64_t)w * h;
        if (!n) return 0;
        img_from_u8<<<blocks_for(n), kImgThreads, 0, st>>>(dst, src, w, h, c);
    }
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_img_to_u8(uint8_t* dst, const float* src, uint32_t w, uint32_t h, uint32_t c,
                                    cudaStream_t st) {
    const uint64_t n = (uint64_t)w * h;
    if (!n) return 0;
    img_to_u8<<<blocks_for(n), kImgThreads, 0, st>>>(dst, src, w, h, c);
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_img_draw_box(float* img, int32_t w, int32_t h, int32_t x1, int32_t y1, int32_t x2, int32_t y2,
                                       int32_t wi, float r, float g, float b, cudaStream_t st) {
    if (wi <= 0) return 0;
    const int32_t span = w > h ? w : h;
    dim3 grid((unsigned)blocks_for((uint64_t)span), (unsigned)(wi < 4096 ? wi : 4096));
    img_draw_box<<<grid, kImgThreads, 0, st>>>(img, w, h, x1, y1, x2, y2, wi, r, g, b);
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_img_draw_text(float* img, int32_t w, int32_t h, const int32_t* glyphs, int32_t n, float r,
                                        float g, float b, cudaStream_t st) {
    if (n <= 0) return 0;
    img_draw_text<<<n, 128, 0, st>>>(img, w, h, glyphs, r, g, b);
    return (int)cudaGetLastError();
}
