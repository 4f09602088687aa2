// The TT-KV write: tokens encoded straight into their paged slots, and the fit tail.
//
//   project_kernel       c = M @ pinv for every token of the layer (frozen projection,
//                        vllm_ttkv/encode.py:301-351), one warp per (token, coefficient)
//   encode_block_kernel  one CTA per (KV head, block of 64 tokens): the per-token int8
//                        quantisation of c, the head's residual R = K - (cq*cs) @ decoder with the
//                        decoder slice staged once per block, then the exact top-k lane select +
//                        quantise + MSB-first pack of the K residual rows and the V rows, written
//                        at the tokens' slots (select_triton.py:157-232); the head-0 CTA also
//                        writes the coefficient blocks and their rulers
//   select_rows_kernel   the same select/pack for caller-supplied (head, token) rows
//   fit-tail kernels     everything build_k_layer (codec/ttkv_packed_cache.py:337-375) does after
//                        the SVDs: coefficient quantisation, core quantisation, the decoder
//                        contraction and its per-row quantisation, zero-padded to the budget
//
// Bit-exactness: given the same fp32 inputs the bytes equal the reference writer's. The rules
// that make that true are each named where they are applied.
#include <cfloat>
#include <cmath>

#include "ttkv_async.cuh"
#include "ttkv_common.cuh"

namespace ttkv {
namespace {

constexpr uint32_t FULL = 0xffffffffu;

// ------------------------------------------------------------------ warp select + pack
// One warp packs one 128-lane row x (lane L of the warp holds lanes 4L..4L+3) into `dst`
// (bitmap d/8 bytes, ceil(lanes*bits/8) code bytes, fp16 ruler). `codes` is 128 bytes of
// per-warp scratch in shared memory, 4-byte aligned: the code stream is assembled there as 32
// big-endian words (stream bit p is bit 31 - p % 32 of word p / 32).
//
// Selection (select_triton.py:180-193): the k-th largest |x| is built one bit at a time on the
// fp32 magnitude bits (monotone for non-negative floats); every lane above it is kept, then the
// lowest-index lanes equal to it until exactly k are kept.
// Ruler (select_triton.py:195-201): max|x| over the row (the largest kept lane), 1 if zero, times
// the fp32 reciprocal of 2^(bits-1)-1. Code: rint(x / ruler) with a correctly rounded division,
// clamped, offset by 2^(bits-1) (select_triton.py:202-203).
__device__ __forceinline__ void warp_select_pack(const float (&x)[4], int lanes, int bits,
                                                 uint8_t* dst, uint8_t* codes) {
    const int L = threadIdx.x & 31;
    uint32_t u[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) u[i] = __float_as_uint(fabsf(x[i]));

    // two bits per step (bits 30..1, then bit 0): the three candidates' counts are independent
    // reductions, and the greedy choice among them equals two one-bit steps (the count of lanes
    // at or above a threshold does not grow with the threshold)
    auto count_ge = [&](uint32_t c) {
        return __reduce_add_sync(FULL, int(u[0] >= c) + int(u[1] >= c) + int(u[2] >= c) + int(u[3] >= c));
    };
    uint32_t t = 0;
    #pragma unroll
    for (int b = 30; b >= 2; b -= 2) {
        const uint32_t c3 = t | (3u << (b - 1)), c2 = t | (2u << (b - 1)), c1 = t | (1u << (b - 1));
        const int n3 = count_ge(c3), n2 = count_ge(c2), n1 = count_ge(c1);
        t = n3 >= lanes ? c3 : n2 >= lanes ? c2 : n1 >= lanes ? c1 : t;
    }
    if (count_ge(t | 1u) >= lanes) t |= 1u;
    const int above_local = int(u[0] > t) + int(u[1] > t) + int(u[2] > t) + int(u[3] > t);
    const int n_above = __reduce_add_sync(FULL, above_local);
    const int tie_local = int(u[0] == t) + int(u[1] == t) + int(u[2] == t) + int(u[3] == t);
    // exclusive prefix of ties over lower warp lanes
    int tie_excl = tie_local;
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(FULL, tie_excl, off);
        if (L >= off) tie_excl += v;
    }
    tie_excl -= tie_local;
    bool sel[4];
    int seen = tie_excl;
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool tie = u[i] == t;
        seen += int(tie);
        sel[i] = (u[i] > t) || (tie && seen <= lanes - n_above);
    }
    const int sel_local = int(sel[0]) + int(sel[1]) + int(sel[2]) + int(sel[3]);
    int rank = sel_local;
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(FULL, rank, off);
        if (L >= off) rank += v;
    }
    rank -= sel_local;                                    // exclusive: rank of this thread's first kept lane

    const uint32_t umax_local = max(max(u[0], u[1]), max(u[2], u[3]));
    const uint32_t umax = __reduce_max_sync(FULL, umax_local);
    const float rmax = __uint_as_float(umax);
    const float sc = __fmul_rn(rmax == 0.f ? 1.f : rmax, inv_ruler(bits));
    const float lo = -float(1 << (bits - 1)), hi = float((1 << (bits - 1)) - 1);
    uint32_t* words = reinterpret_cast<uint32_t*>(codes);
    words[L] = 0u;
    __syncwarp();
    // the k-th kept code occupies stream bits [k * bits, (k + 1) * bits), MSB first; a code that
    // crosses a word boundary is split over the two words
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (sel[i]) {
            float qf = rintf(__fdiv_rn(x[i], sc));
            qf = fminf(fmaxf(qf, lo), hi) + float(1 << (bits - 1));
            const uint32_t c = uint32_t(qf);
            const int pos = rank * bits, wi = pos >> 5, off = pos & 31, spill = off + bits - 32;
            if (spill <= 0) {
                atomicOr(&words[wi], c << (32 - bits - off));
            } else {
                atomicOr(&words[wi], c >> spill);
                atomicOr(&words[wi + 1], c << (32 - spill));
            }
            ++rank;
        }
    }
    // bitmap: lanes 8k..8k+7 live in threads 2k (high nibble) and 2k+1 (low nibble)
    const uint32_t nib = (uint32_t(sel[0]) << 3) | (uint32_t(sel[1]) << 2) | (uint32_t(sel[2]) << 1) |
                         uint32_t(sel[3]);
    const uint32_t other = __shfl_down_sync(FULL, nib, 1);
    if ((L & 1) == 0) dst[L >> 1] = uint8_t((nib << 4) | other);
    __syncwarp();
    // codes: MSB-first stream, row padded to whole bytes (codec/ttkv_packed_cache.py:50-66); byte
    // j of the stream is byte 3 - j % 4 of word j / 4
    const int pb = packed_row_bytes(lanes, bits);
    for (int by = L; by < pb; by += 32)
        dst[16 + by] = uint8_t(words[by >> 2] >> (24 - 8 * (by & 3)));
    if (L == 0) store_f16_bytes(dst + 16 + pb, sc);
    __syncwarp();
}

// ------------------------------------------------------------------ frozen projection
// (the two-launch frozen write, for pools the fused kernel cannot map)
struct ProjParams {
    int H, r1;
    const int64_t* slots;     // skip_pad: a token with a negative slot is not projected
    int skip_pad;
    const void* k;
    int k_dtype;
    int64_t k_stride;
    const int32_t* tok_dec;
    const float* pinvs;       // per decoder: [r1, H*d] (pinv transposed)
    int64_t pinv_stride;
    int n_decoders;
    float* c;                 // [n_tok, r1]
    int32_t* status;
};

constexpr int PROJ_WARPS = 8;

// grid (ceil(r1 / PROJ_WARPS), n_tok): warp w computes coefficient blockIdx.x*8+w of token
// blockIdx.y as a 1024-long dot product over the token's K row (m = h*d + j).
__global__ void __launch_bounds__(PROJ_WARPS * 32) project_kernel(const ProjParams P) {
    const int t = blockIdx.y;
    const int w = threadIdx.x >> 5, L = threadIdx.x & 31;
    const int rr = blockIdx.x * PROJ_WARPS + w;
    const int HD = P.H * kHeadDim;
    __shared__ float m_s[8 * kHeadDim];
    for (int i = threadIdx.x; i < HD; i += blockDim.x)
        m_s[i] = load_elt(P.k, P.k_dtype, int64_t(t) * P.k_stride + i);
    __syncthreads();
    if (P.skip_pad && P.slots[t] < 0) return;                 // a padding token: nothing to write
    const int di = P.tok_dec[t];
    if (di < 0 || di >= P.n_decoders) {
        if (threadIdx.x == 0) report(P.status, TTKV_STATUS_DECODER);
        return;
    }
    if (rr >= P.r1) return;
    const float* pv = P.pinvs + int64_t(di) * P.pinv_stride + int64_t(rr) * HD;
    // four independent partial sums (HD = H*128 is a multiple of 128) keep four loads in flight
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int m = L; m < HD; m += 128) {
        a0 = fmaf(m_s[m], pv[m], a0);
        a1 = fmaf(m_s[m + 32], pv[m + 32], a1);
        a2 = fmaf(m_s[m + 64], pv[m + 64], a2);
        a3 = fmaf(m_s[m + 96], pv[m + 96], a3);
    }
    float acc = (a0 + a1) + (a2 + a3);
    #pragma unroll
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(FULL, acc, off);
    if (L == 0) P.c[int64_t(t) * P.r1 + rr] = acc;
}

// ------------------------------------------------------------------ encode + pack
struct EncParams {
    int H, r1, res_k, res_bits, v_lanes, v_bits, coeff_bytes, k_row, v_row, v_offset;
    int h_lo;                 // the cache holds heads [h_lo, h_lo + gridDim.x): head h's rows are
                              // written at h - h_lo (v_offset is the cache layout's)
    uint8_t* cache;
    int64_t n_slots, row_bytes;
    int skip_pad;             // TTKV_CACHE_SKIP_PAD: a negative slot is skipped, not refused
    const int64_t* slots;
    const void* k;
    int k_dtype;
    int64_t k_stride;
    const void* v;
    int v_dtype;
    int64_t v_stride;
    const int32_t* tok_dec;
    const float* decoders;    // per decoder: [r1, H*d]
    int64_t dec_stride;
    int n_decoders;
    const float* c;           // projected coefficients [n_tok, r1] (frozen path) or null
    const int8_t* coeff_q;    // given codes [n_tok, r1] (fit path)
    const float* coeff_scale; // given rulers [n_tok] fp32 (fit path)
    int32_t* status;
};

// ------------------------------------------------------------------ encode + pack, many tokens a CTA
// The write given the coefficients (the fit path's codes, or the frozen path's projected c),
// computed by CTAs of EB_THREADS threads over blocks of `tb`
// tokens of one KV head (grid: heads written x token blocks). The per-(token, head) form reads the
// head's [r1, 128] fp32 decoder slice once per token from L2 (56 KB at r1 = 110, ~7 GB per layer
// of a 16k-token fit, at 1.1% of HBM); a CTA here stages it in shared memory once for its block (re-staged only
// where the block's tokens change decoder, i.e. cross a request boundary). Per block:
//
//   stage     the decoder slice D [r1][128] and, per token, g[r] = cq * cs (given codes and rulers on
//             the fit path; quantised from the projected c on the frozen path) and the token's checks
//   residual  R[t][j] = K[t][h*128 + j] - sum_r g_t[r] D[r][j], the same four interleaved partial
//             sums as a per-token dot product would take, 8 tokens per pass per thread
//   pack      warp w selects, quantises and packs the K residual rows and the V rows of tokens
//             w, w + 8, ...; the head-0 CTA writes each token's coefficient block and ruler
constexpr int EB_THREADS = 512;
constexpr int EB_WARPS = EB_THREADS / 32;

// Shared memory of encode_block_kernel for r1 and a block of tb tokens.
inline size_t eb_smem(int r1, int tb) {
    return size_t(r1) * 128 * 4 + size_t(r1) * tb * 4 + size_t(tb) * 128 * 4 + size_t(tb) * (4 + 4) +
           size_t(EB_WARPS) * 256 + size_t(tb) * r1 + 64;
}

__global__ void __launch_bounds__(EB_THREADS) encode_block_kernel(const EncParams P, int tb, int n_tok) {
    extern __shared__ __align__(16) unsigned char eb_dyn[];
    const int hs = int(blockIdx.x), h = P.h_lo + hs;
    const int t0 = int(blockIdx.y) * tb;
    const int nb = min(tb, n_tok - t0);
    const int tid = threadIdx.x, w = tid >> 5, L = tid & 31;
    float* D = reinterpret_cast<float*>(eb_dyn);                       // [r1][128]
    float* g = D + P.r1 * 128;                                          // [r1][tb]
    float* R = g + P.r1 * tb;                                           // [tb][128]
    float* cs_s = R + tb * 128;                                         // [tb]
    int* ok_s = reinterpret_cast<int*>(cs_s + tb);                      // [tb] token valid
    uint8_t* codes_s = reinterpret_cast<uint8_t*>(ok_s + tb);          // [warps][2][128]
    int8_t* cq_s = reinterpret_cast<int8_t*>(codes_s + EB_WARPS * 256); // [tb][r1]
    __shared__ int run_end;

    // token checks (every CTA of the token's head group reports the same way)
    for (int tt = tid; tt < nb; tt += EB_THREADS) {
        const int t = t0 + tt;
        const int64_t slot = P.slots[t];
        int ok = 1;
        if (slot < 0 && P.skip_pad) ok = 0;
        else if (slot < 0 || slot >= P.n_slots) { ok = 0; report(P.status, TTKV_STATUS_SLOT_RANGE); }
        const int di = P.tok_dec ? P.tok_dec[t] : 0;
        if (ok && P.decoders && (di < 0 || di >= P.n_decoders)) { ok = 0; report(P.status, TTKV_STATUS_DECODER); }
        ok_s[tt] = ok;
    }
    __syncthreads();

    int staged = -1;                                   // the decoder whose slice D holds
    for (int a = 0; a < nb;) {
        // ---- the run of tokens [a, b) that share a decoder
        if (tid == 0) {
            const int da = P.tok_dec ? P.tok_dec[t0 + a] : 0;
            int b = a + 1;
            while (b < nb && (P.tok_dec ? P.tok_dec[t0 + b] : 0) == da) ++b;
            run_end = b;
        }
        __syncthreads();
        const int b = run_end;
        const int di = P.tok_dec ? P.tok_dec[t0 + a] : 0;
        const bool dec_ok = di >= 0 && di < P.n_decoders;
        if (dec_ok && di != staged) {
            const float4* src = reinterpret_cast<const float4*>(P.decoders + int64_t(di) * P.dec_stride + h * kHeadDim);
            const int64_t rs4 = int64_t(P.H) * kHeadDim / 4;
            for (int i = tid; i < P.r1 * 32; i += EB_THREADS) {
                const int rr = i >> 5, c4 = i & 31;
                reinterpret_cast<float4*>(D)[i] = src[rr * rs4 + c4];
            }
            staged = di;
        }
        // ---- the run's coefficients: g[r][tt] = cq * cs, and the codes for the coefficient block
        if (P.c) {
            // frozen path (vllm_ttkv/encode.py:329-333): a warp per token
            for (int tt = a + w; tt < b; tt += EB_WARPS) {
                const float* c = P.c + int64_t(t0 + tt) * P.r1;
                float amax = 0.f;
                for (int i = L; i < P.r1; i += 32) amax = fmaxf(amax, fabsf(c[i]));
                amax = __uint_as_float(__reduce_max_sync(FULL, __float_as_uint(amax)));
                float cs = __fmul_rn(amax, inv_ruler(8));
                cs = (cs == 0.f) ? 1.f : cs;
                for (int i = L; i < P.r1; i += 32) {
                    const float qf = fminf(fmaxf(rintf(__fdiv_rn(c[i], cs)), -128.f), 127.f);
                    cq_s[tt * P.r1 + i] = int8_t(qf);
                    g[i * tb + tt] = qf * cs;
                }
                if (L == 0) cs_s[tt] = cs;
            }
        } else {
            for (int i = tid; i < (b - a) * P.r1; i += EB_THREADS) {
                const int tt = a + i / P.r1, rr = i - (tt - a) * P.r1;
                const int8_t q = P.coeff_q[int64_t(t0 + tt) * P.r1 + rr];
                const float cs = P.coeff_scale[t0 + tt];
                cq_s[tt * P.r1 + rr] = q;
                g[rr * tb + tt] = float(q) * cs;
                if (rr == 0) cs_s[tt] = cs;
            }
        }
        __syncthreads();

        // ---- residual rows of the run: thread (j, q) takes tokens a + 8 q + 8 * (EB_THREADS / 128) i
        {
            const int j = tid & 127, q = tid >> 7;
            for (int base = a + 8 * q; base < b; base += 8 * (EB_THREADS / 128)) {
                float k0[8], k1[8], k2[8], k3[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) { k0[u] = 0.f; k1[u] = 0.f; k2[u] = 0.f; k3[u] = 0.f; }
                if (P.decoders && dec_ok) {
                    int rr = 0;
                    for (; rr + 4 <= P.r1; rr += 4) {
                        const float d0 = D[rr * 128 + j], d1 = D[(rr + 1) * 128 + j];
                        const float d2 = D[(rr + 2) * 128 + j], d3 = D[(rr + 3) * 128 + j];
                        #pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const int tt = min(base + u, b - 1);
                            k0[u] = fmaf(g[rr * tb + tt], d0, k0[u]);
                            k1[u] = fmaf(g[(rr + 1) * tb + tt], d1, k1[u]);
                            k2[u] = fmaf(g[(rr + 2) * tb + tt], d2, k2[u]);
                            k3[u] = fmaf(g[(rr + 3) * tb + tt], d3, k3[u]);
                        }
                    }
                    for (; rr < P.r1; ++rr) {
                        const float d0 = D[rr * 128 + j];
                        #pragma unroll
                        for (int u = 0; u < 8; ++u) k0[u] = fmaf(g[rr * tb + min(base + u, b - 1)], d0, k0[u]);
                    }
                }
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int tt = base + u;
                    if (tt < b) {
                        const float kv = load_elt(P.k, P.k_dtype, int64_t(t0 + tt) * P.k_stride + h * kHeadDim + j);
                        R[tt * 128 + j] = kv - ((k0[u] + k1[u]) + (k2[u] + k3[u]));
                    }
                }
            }
        }
        __syncthreads();

        // ---- pack: K residual and V rows, a warp per token; the coefficient block once per token
        for (int tt = a + w; tt < b; tt += EB_WARPS) {
            if (!ok_s[tt]) continue;
            const int t = t0 + tt;
            uint8_t* row = P.cache + P.slots[t] * P.row_bytes;
            float x[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = R[tt * 128 + 4 * L + i];
            warp_select_pack(x, P.res_k, P.res_bits, row + P.coeff_bytes + 2 + hs * P.k_row, codes_s + w * 256);
            #pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = load_elt(P.v, P.v_dtype, int64_t(t) * P.v_stride + h * kHeadDim + 4 * L + i);
            warp_select_pack(x, P.v_lanes, P.v_bits, row + P.v_offset + hs * P.v_row, codes_s + w * 256 + 128);
            if (hs == 0) {
                for (int i = L; i < P.r1; i += 32) row[i] = uint8_t(cq_s[tt * P.r1 + i]);
                if (L == 0) store_f16_bytes(row + P.coeff_bytes, cs_s[tt]);
            }
        }
        __syncthreads();
        a = b;
    }
}

// ------------------------------------------------------------------ fused frozen write
// The frozen write of a token in ONE launch: a cluster of H CTAs per token, CTA h = KV head h.
//
//   copy      two 2-D TMA boxes (no multicast) bring this head's 128 columns of the request's
//             transposed pseudo-inverse and of its decoder, r1 rows each, into shared memory;
//             meanwhile warp 7 packs the head's V row and the head's K row is staged
//   project   partial coefficients over this head's columns, c_h[i] = sum_j K[h*d+j] pinvT[i][h*d+j]
//   reduce    c[i] = sum over the cluster's CTAs of c_h[i], read from their shared memory (DSMEM),
//             in rank order, so every CTA holds the same c
//   quantise  cs = amax|c| * fp32(1/127) (0 -> 1), cq = clamp(rint(c / cs))   (encode.py:329-333)
//   residual  R = K - (cq*cs) @ decoder[:, h]                                  (encode.py:335-336)
//   pack      the K residual row; CTA 0 also writes the coefficient block and its ruler
//
// A head-sharded cache holds heads [h_lo, h_hi) only (the storage-sharded format): every CTA of
// the cluster still projects (c needs every head), but only the held heads load their decoder
// slice and write rows, at h - h_lo, and CTA h_lo writes the coefficient block.
//
// Every CTA of a cluster handles the same token, so the early exits (a bad slot or decoder index)
// are taken by all of them together, before the first cluster barrier.
struct FrozenParams {
    int H, r1, res_k, res_bits, v_lanes, v_bits, coeff_bytes, k_row, v_row, v_offset;
    int h_lo, h_hi;           // heads the cache holds: every CTA projects, these write their rows
                              // at h - h_lo (v_offset is the cache layout's)
    uint8_t* cache;
    int64_t n_slots, row_bytes;
    int skip_pad;             // TTKV_CACHE_SKIP_PAD: a negative slot is skipped, not refused
    const int64_t* slots;
    const void* k;
    int k_dtype;
    int64_t k_stride;
    const void* v;
    int v_dtype;
    int64_t v_stride;
    const int32_t* tok_dec;
    int n_decoders;
    int32_t* status;
};

// The decoder pool and the pinv pool as 2-D fp32 tensors [n_decoders * r1 rows, H*d], boxes of
// 128 columns x r1 rows.
struct FrozenMaps {
    CUtensorMap pinv, dec;
};

constexpr int WF_THREADS = 256;
constexpr size_t kFusedWriteSmemMax = 200 * 1024;      // the two slices, r1 <= 200
// The fused write stages both slices once per token, the two-launch write its decoder slice once
// per 64-token block: the fused one is faster up to about a hundred tokens (a decode step's
// batch; B200, r1 = 110, H = 8: 56 vs 72 us at 64 tokens, 97 vs 77 us at 128), the two-launch one
// beyond (a prefill chunk: 215 vs 1421 us at 2048 tokens).
constexpr int32_t kFusedMaxTokens = 96;
constexpr int32_t kMaxGridY = 65535;

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// This CTA's shared-memory word `p` as seen from CTA `rank` of the cluster.
__device__ __forceinline__ float ld_peer(const float* p, int rank) {
    uint32_t a;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}

// grid (H, n_tok), cluster (H, 1, 1), 256 threads; dynamic shared memory 2 * r1 * 512 bytes.
__global__ void __launch_bounds__(WF_THREADS) write_frozen_kernel(const FrozenParams P,
                                                                  const __grid_constant__ FrozenMaps M) {
    extern __shared__ __align__(128) unsigned char wf_dyn[];
    float* pinv_s = reinterpret_cast<float*>(wf_dyn);       // [r1][128]
    float* dec_s = pinv_s + P.r1 * kHeadDim;                 // [r1][128]
    __shared__ __align__(16) float k_s[kHeadDim];
    __shared__ float cpart_s[kMaxRank];                      // read by every CTA of the cluster
    __shared__ float g_s[kMaxRank];
    __shared__ int8_t cq_s[kMaxRank];
    __shared__ float kd_s[2][kHeadDim];
    __shared__ __align__(16) uint8_t codes_s[2][128];
    __shared__ float wmax_s[WF_THREADS / 32];
    __shared__ float cs_s;
    __shared__ __align__(8) uint64_t bar;

    const int h = blockIdx.x, t = blockIdx.y;
    const int tid = threadIdx.x, w = tid >> 5, L = tid & 31;
    pdl_trigger();                                           // the read of the step may launch
    const int64_t slot = P.slots[t];
    if (slot < 0 && P.skip_pad) return;                      // the cluster's token: uniform
    if (slot < 0 || slot >= P.n_slots) {
        if (tid == 0 && h == 0) report(P.status, TTKV_STATUS_SLOT_RANGE);
        return;
    }
    const int di = P.tok_dec[t];
    if (di < 0 || di >= P.n_decoders) {
        if (tid == 0 && h == 0) report(P.status, TTKV_STATUS_DECODER);
        return;
    }
    uint8_t* row = P.cache + slot * P.row_bytes;
    const bool held = h >= P.h_lo && h < P.h_hi;             // this head's rows are written here
    const int hs = h - P.h_lo;

    if (tid == 0) mbar_init(&bar, 1);
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(&bar, uint32_t((held ? 2 : 1) * P.r1 * kHeadDim * sizeof(float)));
        tma_load_2d(pinv_s, &M.pinv, h * kHeadDim, di * P.r1, &bar);
        if (held) tma_load_2d(dec_s, &M.dec, h * kHeadDim, di * P.r1, &bar);
    }
    if (tid < kHeadDim) k_s[tid] = load_elt(P.k, P.k_dtype, int64_t(t) * P.k_stride + h * kHeadDim + tid);
    if (w == 7 && held) {                                    // V needs nothing from the projection
        float x[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i)
            x[i] = load_elt(P.v, P.v_dtype, int64_t(t) * P.v_stride + h * kHeadDim + 4 * L + i);
        warp_select_pack(x, P.v_lanes, P.v_bits, row + P.v_offset + hs * P.v_row, codes_s[1]);
    }
    const bool landed = mbar_wait(&bar, 0);
    const bool bad = __syncthreads_or(!landed);              // also publishes k_s
    if (bad && tid == 0) report(P.status, TTKV_STATUS_TIMEOUT);

    // ---- this head's partial coefficients: warp w takes rows w, w+8, ...
    if (!bad) {
        const float4 kv = reinterpret_cast<const float4*>(k_s)[L];
        for (int i = w; i < P.r1; i += WF_THREADS / 32) {
            const float4 p = reinterpret_cast<const float4*>(pinv_s + i * kHeadDim)[L];
            float a = kv.x * p.x;
            a = fmaf(kv.y, p.y, a);
            a = fmaf(kv.z, p.z, a);
            a = fmaf(kv.w, p.w, a);
            #pragma unroll
            for (int off = 16; off; off >>= 1) a += __shfl_xor_sync(FULL, a, off);
            if (L == 0) cpart_s[i] = a;
        }
    }
    cluster_arrive();
    cluster_wait();                                          // every head's partials are visible

    float c = 0.f;
    if (!bad && tid < P.r1)
        for (int j = 0; j < P.H; ++j) c += ld_peer(&cpart_s[tid], j);
    cluster_arrive();                                        // done reading the peers (waited at exit)

    // ---- quantise the coefficients (every CTA, identical inputs -> identical codes)
    float a = __uint_as_float(__reduce_max_sync(FULL, __float_as_uint(fabsf(c))));
    if (L == 0) wmax_s[w] = a;
    __syncthreads();
    if (tid == 0) {
        float amax = wmax_s[0];
        #pragma unroll
        for (int i = 1; i < WF_THREADS / 32; ++i) amax = fmaxf(amax, wmax_s[i]);
        const float cs = __fmul_rn(amax, inv_ruler(8));
        cs_s = (cs == 0.f) ? 1.f : cs;
    }
    __syncthreads();
    const float cs = cs_s;
    if (tid < P.r1) {
        const float qf = fminf(fmaxf(rintf(__fdiv_rn(c, cs)), -128.f), 127.f);
        cq_s[tid] = int8_t(qf);
        g_s[tid] = qf * cs;
    }
    __syncthreads();

    // ---- (cq*cs) @ decoder[:, h]: the two thread halves take the two halves of the rows
    if (!bad && held) {
        const int half = tid >> 7, j = tid & 127;
        const int mid = (P.r1 + 1) >> 1;
        const int i0 = half ? mid : 0, i1 = half ? P.r1 : mid;
        float k0 = 0.f, k1 = 0.f, k2 = 0.f, k3 = 0.f;
        int i = i0;
        for (; i + 4 <= i1; i += 4) {
            k0 = fmaf(g_s[i], dec_s[i * kHeadDim + j], k0);
            k1 = fmaf(g_s[i + 1], dec_s[(i + 1) * kHeadDim + j], k1);
            k2 = fmaf(g_s[i + 2], dec_s[(i + 2) * kHeadDim + j], k2);
            k3 = fmaf(g_s[i + 3], dec_s[(i + 3) * kHeadDim + j], k3);
        }
        for (; i < i1; ++i) k0 = fmaf(g_s[i], dec_s[i * kHeadDim + j], k0);
        kd_s[half][j] = (k0 + k1) + (k2 + k3);
    }
    __syncthreads();

    if (!bad && held && w == 0) {
        float x[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = k_s[4 * L + i] - (kd_s[0][4 * L + i] + kd_s[1][4 * L + i]);
        warp_select_pack(x, P.res_k, P.res_bits, row + P.coeff_bytes + 2 + hs * P.k_row, codes_s[0]);
    } else if (!bad && w == 1 && h == P.h_lo) {
        for (int i = L; i < P.r1; i += 32) row[i] = uint8_t(cq_s[i]);
        if (L == 0) store_f16_bytes(row + P.coeff_bytes, cs);
    }
    cluster_wait();                                          // no CTA leaves while a peer reads it
    if (bad) mbar_wait(&bar, 0);                             // let late copies land (bounded) first
}

// ------------------------------------------------------------------ standalone rows
struct RowsParams {
    uint8_t* cache;
    int64_t n_slots, row_bytes;
    int skip_pad;             // TTKV_CACHE_SKIP_PAD: a negative slot is skipped, not refused
    const int64_t* slots;
    int n_tok, heads, field_off, row_stride, lanes, bits;
    const void* x;
    int x_dtype;
    int32_t* status;
};

// 4 rows per CTA, one warp each; row i = h*n_tok + t (select_triton.py:173-177).
__global__ void __launch_bounds__(128) select_rows_kernel(const RowsParams P) {
    __shared__ __align__(16) uint8_t codes_s[4][128];
    const int w = threadIdx.x >> 5, L = threadIdx.x & 31;
    const int64_t i = int64_t(blockIdx.x) * 4 + w;
    if (i >= int64_t(P.n_tok) * P.heads) return;
    const int t = int(i % P.n_tok), h = int(i / P.n_tok);
    const int64_t slot = P.slots[t];
    if (slot < 0 && P.skip_pad) return;
    if (slot < 0 || slot >= P.n_slots) {
        if (L == 0) report(P.status, TTKV_STATUS_SLOT_RANGE);
        return;
    }
    float x[4];
    #pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = load_elt(P.x, P.x_dtype, i * kHeadDim + 4 * L + k);
    warp_select_pack(x, P.lanes, P.bits, P.cache + slot * P.row_bytes + P.field_off + h * P.row_stride,
                     codes_s[w]);
}

// ------------------------------------------------------------------ fit tail
// Per-token coefficient quantisation of the token core G1 [n, r] (ttkv_packed_cache.py:353-356):
// cs = amax * fp32(1/127), 0 -> 1, cq = clamp(rint(c/cs)); codes zero-padded to `budget`.
__global__ void __launch_bounds__(32) quant_coeff_kernel(const float* G1, int n, int r, int budget,
                                                         int8_t* cq, float* cs_out) {
    const int t = blockIdx.x, L = threadIdx.x;
    float a = 0.f;
    for (int i = L; i < r; i += 32) a = fmaxf(a, fabsf(G1[int64_t(t) * r + i]));
    a = __uint_as_float(__reduce_max_sync(FULL, __float_as_uint(a)));
    float cs = __fmul_rn(a, inv_ruler(8));
    cs = cs == 0.f ? 1.f : cs;
    for (int i = L; i < budget; i += 32) {
        float qf = 0.f;
        if (i < r) qf = fminf(fmaxf(rintf(__fdiv_rn(G1[int64_t(t) * r + i], cs)), -128.f), 127.f);
        cq[int64_t(t) * budget + i] = int8_t(qf);
    }
    if (L == 0) cs_out[t] = cs;
}

// quant_cores (codec/ttkv_codec.py:142-163): per row s = max(amax, 1e-12) * fp32(1/127),
// out = clamp(rint(M/s), -127, 127) * s.
__global__ void __launch_bounds__(32) quant_core_rows_kernel(const float* M, int cols, float* out) {
    const int row = blockIdx.x, L = threadIdx.x;
    const float* m = M + int64_t(row) * cols;
    float a = 0.f;
    for (int i = L; i < cols; i += 32) a = fmaxf(a, fabsf(m[i]));
    a = __uint_as_float(__reduce_max_sync(FULL, __float_as_uint(a)));
    const float s = __fmul_rn(fmaxf(a, 1e-12f), inv_ruler(8));
    for (int i = L; i < cols; i += 32)
        out[int64_t(row) * cols + i] = fminf(fmaxf(rintf(__fdiv_rn(m[i], s)), -127.f), 127.f) * s;
}

// dec[a, h*d + j] = sum_b G2q[a, j, b] * G3q[b, h]   ("ajb,bh->ahj", ttkv_packed_cache.py:361)
__global__ void decoder_contract_kernel(const float* G2q, const float* G3q, int r2, int H, int d,
                                        float* dec) {
    const int a = blockIdx.x;
    for (int m = threadIdx.x; m < H * d; m += blockDim.x) {
        const int h = m / d, j = m % d;
        float acc = 0.f;
        for (int b = 0; b < r2; ++b)
            acc = fmaf(G2q[(int64_t(a) * d + j) * r2 + b], G3q[b * H + h], acc);
        dec[int64_t(a) * H * d + m] = acc;
    }
}

// _quant_rows (ttkv_packed_cache.py:170-176) of the decoder and its fp32 form
// decoder_f = dec_q * fp16(scale) (ttkv_packed_cache.py:290-293), rows past r zero.
__global__ void __launch_bounds__(256) decoder_quant_kernel(const float* dec, int r, int budget, int cols,
                                                            int8_t* dec_q, uint16_t* dec_scale,
                                                            float* decoder) {
    const int a = blockIdx.x;
    __shared__ float wmax[8];
    __shared__ float sc_s;
    if (a >= r) {
        for (int i = threadIdx.x; i < cols; i += blockDim.x) decoder[int64_t(a) * cols + i] = 0.f;
        return;
    }
    float m = 0.f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, fabsf(dec[int64_t(a) * cols + i]));
    m = __uint_as_float(__reduce_max_sync(FULL, __float_as_uint(m)));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float rmax = 0.f;
        for (int i = 0; i < int(blockDim.x >> 5); ++i) rmax = fmaxf(rmax, wmax[i]);
        sc_s = __fmul_rn(rmax == 0.f ? 1.f : rmax, inv_ruler(8));
    }
    __syncthreads();
    const float sc = sc_s;
    const uint32_t sh = f16_bits(sc);
    const float sf = f16_bits_to_f32(sh);
    for (int i = threadIdx.x; i < cols; i += blockDim.x) {
        const float qf = fminf(fmaxf(rintf(__fdiv_rn(dec[int64_t(a) * cols + i], sc)), -128.f), 127.f);
        dec_q[int64_t(a) * cols + i] = int8_t(qf);
        decoder[int64_t(a) * cols + i] = qf * sf;
    }
    if (threadIdx.x == 0) dec_scale[a] = uint16_t(sh);
}

int check_cache(const ttkv_cache_t* cache, int need) {
    if (!cache || !cache->base) return fail(TTKV_ERR_ARG, "cache is null");
    if (cache->row_bytes < need || cache->n_slots < 0)
        return fail(TTKV_ERR_ARG, "cache rows are %lld bytes, %d needed", (long long)cache->row_bytes, need);
    return TTKV_OK;
}

// The fused frozen write when the pools map as 2-D TMA tensors and the slices fit in shared
// memory: returns 0 when launched, a negative error code, or 1 to take the two-launch path.
int launch_frozen_fused(const ttkv_layout_t* lay, const ttkv_layout_t* out, int h_lo,
                        const ttkv_cache_t* cache, const int64_t* slots,
                        int32_t n_tok, const void* k, int32_t k_dtype, int64_t k_stride, const void* v,
                        int32_t v_dtype, int64_t v_stride, const int32_t* tok_dec, const float* decoders,
                        int64_t dec_stride, const float* pinvs, int64_t pinv_stride, int32_t n_decoders,
                        int32_t* status, cudaStream_t st) {
    const int64_t cols = int64_t(lay->H) * kHeadDim;
    const size_t dyn = size_t(2) * lay->r1 * kHeadDim * sizeof(float);
    if (lay->H > 8 || dec_stride != lay->r1 * cols || pinv_stride != lay->r1 * cols ||
        (reinterpret_cast<uintptr_t>(decoders) & 15) || (reinterpret_cast<uintptr_t>(pinvs) & 15) ||
        dyn > kFusedWriteSmemMax)
        return 1;
    FrozenMaps maps;
    const uint64_t rows = uint64_t(n_decoders) * lay->r1;
    if (!encode_2d(&maps.pinv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pinvs, cols, rows, cols * 4, kHeadDim,
                   lay->r1, 0) ||
        !encode_2d(&maps.dec, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, decoders, cols, rows, cols * 4, kHeadDim,
                   lay->r1, 0))
        return 1;
    if (raise_smem_limit(reinterpret_cast<const void*>(write_frozen_kernel), "write_frozen_kernel") != TTKV_OK) {
        set_error("%s", "");                                 // the two-launch write serves instead
        return 1;
    }
    {   // the H CTAs of a cluster must fit on the GPU at once (asked once per shape)
        static int last_h = -1;
        static size_t last_dyn = 0;
        static bool last_ok = false;
        if (lay->H != last_h || dyn != last_dyn) {
            cudaLaunchConfig_t q{};
            q.gridDim = dim3(lay->H, 1);
            q.blockDim = dim3(WF_THREADS);
            q.dynamicSmemBytes = dyn;
            cudaLaunchAttribute qa[1];
            qa[0].id = cudaLaunchAttributeClusterDimension;
            qa[0].val.clusterDim.x = lay->H;
            qa[0].val.clusterDim.y = 1;
            qa[0].val.clusterDim.z = 1;
            q.attrs = qa;
            q.numAttrs = 1;
            int n = 0;
            last_ok = cudaOccupancyMaxActiveClusters(&n, write_frozen_kernel, &q) == cudaSuccess && n > 0;
            cudaGetLastError();
            last_h = lay->H;
            last_dyn = dyn;
        }
        if (!last_ok) return 1;
    }
    FrozenParams P{};
    P.H = lay->H; P.r1 = lay->r1; P.res_k = lay->res_k; P.res_bits = lay->res_bits;
    P.v_lanes = lay->v_lanes; P.v_bits = lay->v_bits; P.coeff_bytes = lay->coeff_bytes;
    P.k_row = lay->k_row_bytes; P.v_row = lay->v_row_bytes; P.v_offset = out->v_offset;
    P.h_lo = h_lo; P.h_hi = h_lo + out->H;
    P.cache = cache->base; P.n_slots = cache->n_slots; P.row_bytes = cache->row_bytes;
    P.skip_pad = cache->flags & TTKV_CACHE_SKIP_PAD;
    P.k_dtype = k_dtype; P.k_stride = k_stride; P.v_dtype = v_dtype; P.v_stride = v_stride;
    P.n_decoders = n_decoders; P.status = status;
    const int esz_k = k_dtype == TTKV_F32 ? 4 : 2, esz_v = v_dtype == TTKV_F32 ? 4 : 2;
    for (int32_t t0 = 0; t0 < n_tok; t0 += kMaxGridY) {      // grid.y is at most 65535 tokens
        const int32_t nt = n_tok - t0 < kMaxGridY ? n_tok - t0 : kMaxGridY;
        P.slots = slots + t0;
        P.tok_dec = tok_dec + t0;
        P.k = static_cast<const char*>(k) + int64_t(t0) * k_stride * esz_k;
        P.v = static_cast<const char*>(v) + int64_t(t0) * v_stride * esz_v;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(lay->H, nt);
        cfg.blockDim = dim3(WF_THREADS);
        cfg.dynamicSmemBytes = dyn;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = lay->H;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, write_frozen_kernel, P, maps);
        if (e != cudaSuccess) return fail(TTKV_ERR_CUDA, "write_frozen_kernel: %s", cudaGetErrorString(e));
    }
    return 0;
}

}  // namespace
}  // namespace ttkv

using namespace ttkv;

extern "C" size_t ttkv_write_workspace_bytes(const ttkv_layout_t* lay, int32_t n_tok) {
    if (!lay || n_tok <= 0) return 0;
    return size_t(n_tok) * lay->r1 * sizeof(float);
}

extern "C" int ttkv_write_paged_shard(const ttkv_layout_t* lay, int32_t h_lo, int32_t h_hi,
                                      const ttkv_cache_t* cache, const int64_t* slot_mapping,
                                      int32_t n_tok, const void* k, int32_t k_dtype, int64_t k_stride,
                                      const void* v, int32_t v_dtype, int64_t v_stride,
                                      const int32_t* tok_dec, const float* decoders, int64_t dec_stride,
                                      const float* pinvs, int64_t pinv_stride, int32_t n_decoders,
                                      const int8_t* coeff_q, const float* coeff_scale, void* workspace,
                                      size_t workspace_bytes, int32_t* status, void* stream) {
    if (!lay) return fail(TTKV_ERR_ARG, "layout is null");
    if (lay->d != kHeadDim) return fail(TTKV_ERR_UNSUPPORTED, "head dim %d: d=128 only", lay->d);
    if (lay->qbits != 8) return fail(TTKV_ERR_UNSUPPORTED, "qbits=%d: coefficients are int8", lay->qbits);
    if (lay->r1 > kMaxRank) return fail(TTKV_ERR_UNSUPPORTED, "r1=%d > %d", lay->r1, kMaxRank);
    if (lay->H > 8) return fail(TTKV_ERR_UNSUPPORTED, "H=%d > 8 KV heads", lay->H);
    if (lay->res_k < 1 || lay->res_bits < 2 || lay->v_bits < 2 || lay->res_bits > 8 || lay->v_bits > 8)
        return fail(TTKV_ERR_UNSUPPORTED, "lane widths res_k=%d res_bits=%d v_bits=%d", lay->res_k,
                    lay->res_bits, lay->v_bits);
    if (h_lo < 0 || h_hi > lay->H || h_lo >= h_hi)
        return fail(TTKV_ERR_ARG, "held heads [%d, %d) outside the layout's %d", h_lo, h_hi, lay->H);
    // the cache's rows: the layout of the held heads (the same widths, H = h_hi - h_lo)
    ttkv_layout_t out{};
    if (int e = ttkv_layout_init(&out, h_hi - h_lo, lay->d, lay->r1, lay->qbits, lay->res_k,
                                 lay->res_bits, lay->v_lanes, lay->v_bits, lay->align))
        return e;
    if (int e = check_cache(cache, out.blob_bytes)) return e;
    if (n_tok < 0) return fail(TTKV_ERR_ARG, "n_tok < 0");
    if (n_tok == 0) return TTKV_OK;
    if (!slot_mapping || !k || !v) return fail(TTKV_ERR_ARG, "slot_mapping/k/v null");
    if (k_dtype < TTKV_F32 || k_dtype > TTKV_BF16 || v_dtype < TTKV_F32 || v_dtype > TTKV_BF16)
        return fail(TTKV_ERR_ARG, "k/v dtype");
    if (k_stride < int64_t(lay->H) * 128 || v_stride < int64_t(lay->H) * 128)
        return fail(TTKV_ERR_ARG, "k/v stride below H*d");
    const bool frozen = pinvs != nullptr;
    if (!decoders || !tok_dec || n_decoders < 1) return fail(TTKV_ERR_ARG, "decoders/tok_dec missing");
    if (dec_stride < int64_t(lay->r1) * lay->H * 128) return fail(TTKV_ERR_ARG, "decoder stride");
    if (frozen && pinv_stride < int64_t(lay->r1) * lay->H * 128) return fail(TTKV_ERR_ARG, "pinv stride");
    if (!frozen && (!coeff_q || !coeff_scale)) return fail(TTKV_ERR_ARG, "coeff_q/coeff_scale null");
    if (frozen && (!workspace || workspace_bytes < ttkv_write_workspace_bytes(lay, n_tok)))
        return fail(TTKV_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes,
                    ttkv_write_workspace_bytes(lay, n_tok));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (frozen && n_tok <= kFusedMaxTokens) {
        const int r = launch_frozen_fused(lay, &out, h_lo, cache, slot_mapping, n_tok, k, k_dtype, k_stride,
                                          v, v_dtype, v_stride, tok_dec, decoders, dec_stride, pinvs,
                                          pinv_stride, n_decoders, status, st);
        if (r <= 0) return r;                                // launched (0) or failed (< 0)
    }
    float* c = nullptr;
    if (frozen) {
        ProjParams pp{};
        pp.H = lay->H; pp.r1 = lay->r1; pp.slots = slot_mapping; pp.skip_pad = cache->flags & TTKV_CACHE_SKIP_PAD;
        pp.k = k; pp.k_dtype = k_dtype; pp.k_stride = k_stride;
        pp.tok_dec = tok_dec; pp.pinvs = pinvs; pp.pinv_stride = pinv_stride; pp.n_decoders = n_decoders;
        c = reinterpret_cast<float*>(workspace);
        pp.c = c; pp.status = status;
        dim3 grid((lay->r1 + PROJ_WARPS - 1) / PROJ_WARPS, n_tok);
        project_kernel<<<grid, PROJ_WARPS * 32, 0, st>>>(pp);
        if (int e = check_launch("project_kernel")) return e;
    }
    EncParams ep{};
    ep.H = lay->H; ep.r1 = lay->r1; ep.res_k = lay->res_k; ep.res_bits = lay->res_bits;
    ep.v_lanes = lay->v_lanes; ep.v_bits = lay->v_bits; ep.coeff_bytes = lay->coeff_bytes;
    ep.k_row = lay->k_row_bytes; ep.v_row = lay->v_row_bytes; ep.v_offset = out.v_offset;
    ep.h_lo = h_lo;
    ep.cache = cache->base; ep.n_slots = cache->n_slots; ep.row_bytes = cache->row_bytes;
    ep.skip_pad = cache->flags & TTKV_CACHE_SKIP_PAD;
    ep.slots = slot_mapping; ep.k = k; ep.k_dtype = k_dtype; ep.k_stride = k_stride;
    ep.v = v; ep.v_dtype = v_dtype; ep.v_stride = v_stride; ep.tok_dec = tok_dec;
    ep.decoders = decoders; ep.dec_stride = dec_stride; ep.n_decoders = n_decoders;
    ep.c = c; ep.coeff_q = frozen ? nullptr : coeff_q; ep.coeff_scale = frozen ? nullptr : coeff_scale;
    ep.status = status;
    // blocks of 64 tokens, or 32 where the staged decoder slice leaves too little shared memory
    const int tb = eb_smem(lay->r1, 64) <= 160 * 1024 ? 64 : 32;
    const size_t smem = eb_smem(lay->r1, tb);
    if (int e = raise_smem_limit(reinterpret_cast<const void*>(encode_block_kernel), "encode_block_kernel")) return e;
    encode_block_kernel<<<dim3(h_hi - h_lo, (n_tok + tb - 1) / tb), EB_THREADS, smem, st>>>(ep, tb, n_tok);
    return check_launch("encode_block_kernel");
}

extern "C" int ttkv_write_paged(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                                const int64_t* slot_mapping, int32_t n_tok, const void* k,
                                int32_t k_dtype, int64_t k_stride, const void* v, int32_t v_dtype,
                                int64_t v_stride, const int32_t* tok_dec, const float* decoders,
                                int64_t dec_stride, const float* pinvs, int64_t pinv_stride,
                                int32_t n_decoders, const int8_t* coeff_q, const float* coeff_scale,
                                void* workspace, size_t workspace_bytes, int32_t* status,
                                void* stream) {
    if (!lay) return fail(TTKV_ERR_ARG, "layout is null");
    return ttkv_write_paged_shard(lay, 0, lay->H, cache, slot_mapping, n_tok, k, k_dtype, k_stride, v,
                                  v_dtype, v_stride, tok_dec, decoders, dec_stride, pinvs, pinv_stride,
                                  n_decoders, coeff_q, coeff_scale, workspace, workspace_bytes, status,
                                  stream);
}

extern "C" int ttkv_select_pack_rows(const ttkv_cache_t* cache, const int64_t* slots, int32_t n_tok,
                                     const void* x, int32_t x_dtype, int32_t heads, int32_t d,
                                     int32_t field_off, int32_t row_stride, int32_t lanes,
                                     int32_t bits, int32_t* status, void* stream) {
    if (d != kHeadDim) return fail(TTKV_ERR_UNSUPPORTED, "d=%d: rows of 128 lanes only", d);
    if (lanes < 1 || lanes > d || bits < 2 || bits > 8)
        return fail(TTKV_ERR_UNSUPPORTED, "lanes=%d bits=%d outside 1..d / 2..8", lanes, bits);
    if (heads < 1 || n_tok < 0 || field_off < 0 || row_stride < 0) return fail(TTKV_ERR_ARG, "shape");
    const int need = field_off + (heads - 1) * row_stride + d / 8 + packed_row_bytes(lanes, bits) + 2;
    if (int e = check_cache(cache, need)) return e;
    if (n_tok == 0) return TTKV_OK;
    if (!slots || !x) return fail(TTKV_ERR_ARG, "slots/x null");
    if (x_dtype < TTKV_F32 || x_dtype > TTKV_BF16) return fail(TTKV_ERR_ARG, "x dtype");
    RowsParams p{};
    p.cache = cache->base; p.n_slots = cache->n_slots; p.row_bytes = cache->row_bytes;
    p.skip_pad = cache->flags & TTKV_CACHE_SKIP_PAD;
    p.slots = slots; p.n_tok = n_tok; p.heads = heads; p.field_off = field_off;
    p.row_stride = row_stride; p.lanes = lanes; p.bits = bits; p.x = x; p.x_dtype = x_dtype;
    p.status = status;
    const int64_t rows = int64_t(n_tok) * heads;
    select_rows_kernel<<<unsigned((rows + 3) / 4), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return check_launch("select_rows_kernel");
}

extern "C" size_t ttkv_fit_tail_scratch_bytes(int32_t r, int32_t r2, int32_t H, int32_t d) {
    if (r < 1 || r2 < 1 || H < 1 || d < 1) return 0;
    return (size_t(r) * d * r2 + size_t(r2) * H + size_t(r) * H * d) * sizeof(float);
}

extern "C" int ttkv_fit_tail(const float* G1, const float* G2, const float* G3, int32_t n, int32_t r,
                             int32_t r2, int32_t H, int32_t d, int32_t qbits, int32_t budget,
                             int8_t* coeff_q, float* coeff_scale, int8_t* dec_q, uint16_t* dec_scale,
                             float* decoder, void* scratch, size_t scratch_bytes, void* stream) {
    if (qbits != 8) return fail(TTKV_ERR_UNSUPPORTED, "qbits=%d: the fit tail quantises to int8", qbits);
    if (!G1 || !G2 || !G3 || !coeff_q || !coeff_scale || !dec_q || !dec_scale || !decoder)
        return fail(TTKV_ERR_ARG, "null pointer");
    if (n < 1 || r < 1 || r2 < 1 || H < 1 || d < 1 || budget < r)
        return fail(TTKV_ERR_ARG, "shape n=%d r=%d r2=%d H=%d d=%d budget=%d", n, r, r2, H, d, budget);
    if (!scratch || scratch_bytes < ttkv_fit_tail_scratch_bytes(r, r2, H, d))
        return fail(TTKV_ERR_WORKSPACE, "scratch %zu < %zu bytes", scratch_bytes,
                    ttkv_fit_tail_scratch_bytes(r, r2, H, d));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* G2q = reinterpret_cast<float*>(scratch);
    float* G3q = G2q + size_t(r) * d * r2;
    float* dec = G3q + size_t(r2) * H;
    quant_coeff_kernel<<<n, 32, 0, st>>>(G1, n, r, budget, coeff_q, coeff_scale);
    if (int e = check_launch("quant_coeff_kernel")) return e;
    quant_core_rows_kernel<<<r, 32, 0, st>>>(G2, d * r2, G2q);
    if (int e = check_launch("quant_core_rows_kernel(G2)")) return e;
    quant_core_rows_kernel<<<r2, 32, 0, st>>>(G3, H, G3q);
    if (int e = check_launch("quant_core_rows_kernel(G3)")) return e;
    decoder_contract_kernel<<<r, 256, 0, st>>>(G2q, G3q, r2, H, d, dec);
    if (int e = check_launch("decoder_contract_kernel")) return e;
    decoder_quant_kernel<<<budget, 256, 0, st>>>(dec, r, budget, H * d, dec_q, dec_scale, decoder);
    return check_launch("decoder_quant_kernel");
}
