// Shared device helpers for the TT-KV sm_100a kernels: slot-field access, element loads, the
// packed-row decode and the error plumbing of the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ttkv_b200.h"

namespace ttkv {

constexpr int kHeadDim = 128;     // the only head dim the backend serves (d == 128)
constexpr int kMaxRank = 256;     // largest r1 the kernels accept
constexpr int kMaxG = 8;          // largest GQA group (HQ / H)

// ------------------------------------------------------------------ host error plumbing
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
// Raise a kernel's dynamic shared-memory limit to the device's opt-in maximum (less its static
// shared memory), once per kernel and device; a launch then only names its own size. A per-launch
// limit would be a property of the last launch, not of each launch (a graph node replayed on its
// own, or two threads, would see another layer's value).
int raise_smem_limit(const void* kernel, const char* what);

// ------------------------------------------------------------------ device status
// First error wins: a status word that already holds a code keeps it.
__device__ __forceinline__ void report(int32_t* status, int32_t code) {
    if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------ element loads
__device__ __forceinline__ float load_elt(const void* p, int dtype, int64_t i) {
    if (dtype == TTKV_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    if (dtype == TTKV_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elt(void* p, int dtype, int64_t i, float v) {
    if (dtype == TTKV_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (dtype == TTKV_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// fp32 -> IEEE fp16 bit pattern (round to nearest even), zero-extended into a 32-bit integer
// register inside the asm. Splitting the bits into bytes from a 16-bit half-typed register is
// not safe: a byte store from such a register was compiled as a numeric f16 -> u8 conversion
// (the low byte came out as the truncated value, e.g. 0x01 for 1.24), so the bit pattern only
// ever leaves this function as a plain u32.
__device__ __forceinline__ uint32_t f16_bits(float x) {
    uint32_t r;
    asm("{\n\t.reg .b16 h;\n\tcvt.rn.f16.f32 h, %1;\n\tcvt.u32.u16 %0, h;\n\t}" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
    float x;
    asm("{\n\t.reg .b16 h;\n\tcvt.u16.u32 h, %1;\n\tcvt.f32.f16 %0, h;\n\t}" : "=f"(x) : "r"(bits));
    return x;
}

// An fp16 stored as two little-endian bytes at any (possibly odd) byte offset
// (vllm_ttkv/layout.py:181,191 write `scale.view(uint8)`).
__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return f16_bits_to_f32(uint32_t(p[0]) | (uint32_t(p[1]) << 8));
}

__device__ __forceinline__ void store_f16_bytes(uint8_t* p, float x) {
    const uint32_t b = f16_bits(x);
    p[0] = uint8_t(b & 0xffu);
    p[1] = uint8_t((b >> 8) & 0xffu);
}

// 32 lanes of an MSB-first bitmap as one word with lane l at bit 31-l: bytes are read in
// order and the first byte lands in the top bits (lane 8j+b is bit 7-b of byte j,
// codec/ttkv_packed_cache.py:233-240).
__device__ __forceinline__ uint32_t bitmap_word(const uint8_t* bm, int w) {
    const uint8_t* b = bm + 4 * w;
    return (uint32_t(b[0]) << 24) | (uint32_t(b[1]) << 16) | (uint32_t(b[2]) << 8) | uint32_t(b[3]);
}

// Code of rank `rank` in an MSB-first stream of `bits`-wide codes (codec/ttkv_packed_cache.py:
// 50-66). Reads the byte holding the code's first bit and the next one; when the code fits in
// the first byte the second byte is shifted out, so reading one byte past the stream (the row's
// ruler follows it) never changes the value.
__device__ __forceinline__ int code_at(const uint8_t* stream, int rank, int bits) {
    const int bit = rank * bits;
    const int byte = bit >> 3, sh = bit & 7;
    const uint32_t w = (uint32_t(stream[byte]) << 8) | uint32_t(stream[byte + 1]);
    return int((w >> (16 - sh - bits)) & ((1u << bits) - 1));
}

// Lane j's value in one packed row: (code - 2^(bits-1)) * ruler if lane j is kept, else 0.
// `words` = the row's 4 bitmap words (bitmap_word), `stream` its code bytes, `ruler` fp32.
// (codec/ttkv_packed_cache.py:247-271, PackedRows.materialise.)
__device__ __forceinline__ float lane_value(const uint32_t words[4], const uint8_t* stream,
                                            float ruler, int bits, int j) {
    const int w = j >> 5, l = j & 31;
    const uint32_t word = words[w];
    if (!((word >> (31 - l)) & 1u)) return 0.f;
    int rank = __popc(word & ~(0xffffffffu >> l));
    #pragma unroll
    for (int i = 0; i < 4; ++i) rank += (i < w) ? __popc(words[i]) : 0;
    const int code = code_at(stream, rank, bits) - (1 << (bits - 1));
    return float(code) * ruler;
}

// fp32 reciprocal of the ruler divisor 2^(bits-1)-1, the multiplier torch's CUDA kernel applies
// for `tensor / python_int` (vllm_ttkv/select_triton.py:76-84, :119): a correctly rounded
// fp32 quotient 1/divisor.
__device__ __forceinline__ float inv_ruler(int bits) {
    return __fdiv_rn(1.0f, float((1 << (bits - 1)) - 1));
}

__host__ __device__ inline int packed_row_bytes(int k, int bits) { return (k * bits + 7) / 8; }

}  // namespace ttkv
