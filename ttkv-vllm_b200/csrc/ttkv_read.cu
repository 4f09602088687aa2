// The TT-KV read: decode and chunked-prefill continuation over a paged, packed cache.
//
// One launch covers every request of a layer. A CTA owns (request, KV head, query block, token
// split); it stages its head's slice of the request's decoder in shared memory once and then
// walks 32-token tiles of the request's rows through the block table:
//
//   gather     the tile's slot ids from the block table, the coefficient block, this head's K
//              residual row and V row, and the RoPE rows of the tokens' positions
//   rebuild    K_pre = (cq * cs) @ decoder[:, head]        fp32 FMA (the reference's ieee dot)
//   patch      K_pre += residual lanes (bitmap + MSB-first codes + fp16 ruler)
//   rotate     y = RoPE(K_pre, the row's own position), (j, j + d/2) pairing
//   score      s = scale * q . y for the G query heads (x query block), causal mask
//   softmax    online (running max and sum per query row)
//   readout    o += p * V lanes decoded from the slot
//
// and writes (o, max, sum) per split; a merge kernel combines the splits into the output.
// This is vllm_ttkv/impl.py:511-540 (_decode_one) + krt_triton.py:66-151 (_krt_kernel) +
// softmax + v_out_triton.py:51-118 (_v_out_kernel) for the decode, and impl.py:725-778 with
// krt_triton.py:155-266 / v_out_triton.py:159-246 for the continuation, fused and batched.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <cstring>
#include <cmath>
#include <mutex>

#include "ttkv_async.cuh"
#include "ttkv_common.cuh"

namespace ttkv {
namespace {

constexpr int TT = 32;    // tokens per tile
constexpr int NT = 128;   // threads per CTA
constexpr int RS = 132;   // row stride (floats) of the rotated-key tile

struct ReadParams {
    int H, r1, res_k, res_bits, v_lanes, v_bits, coeff_bytes, k_row, v_row, v_offset, k_pb, v_pb;
    const uint8_t* cache;
    int64_t n_slots, row_bytes;
    int block_size;
    const int32_t* block_table;
    int64_t bt_stride;
    int bt_cols;
    const int32_t* seq_lens;
    const float* decoders;
    int64_t dec_stride;
    const int32_t* dec_index;
    int n_decoders;
    const unsigned char* dec_image;   // optional: ttkv_decoder_image's operand images
    int64_t image_stride;
    const float* dec_scales;
    const void* table;
    int table_dtype;
    int64_t table_rows;
    const void* q;
    int q_dtype;
    int64_t q_stride;
    int HQ, G;
    const int32_t* q_start;   // null for decode
    const int32_t* q_len;
    float scale;
    int head_lo, n_heads;     // KV heads [head_lo, head_lo + n_heads)
    int qmax, n_qblk, n_splits, chunk;
    int n_reqs, n_ctas;       // tensor-core decode: requests, CTAs of the balanced schedule
    int max_seq;              // the call's max_seq_len: a longer request is refused on the device
    int64_t n_part_slots;     // tensor-core decode: partial slots the workspace holds
    // tensor-core decode of continuation chunks (null for a decode): request r of the launch is a
    // block of v_nq[r] consecutive (query, query head) rows of stored request v_req[r], numbered
    // query-major from v_f0[r]: row i is query j = (v_f0 + i) / g_real, head (v_f0 + i) % g_real,
    // at query row v_qrow[r] + j and position v_pos[r] + j, seeing the stored rows before it + 1
    const int32_t* v_req;
    const int32_t* v_qrow;
    const int32_t* v_nq;
    const int32_t* v_pos;
    const int32_t* v_f0;
    int g_real;
    float* part_o;            // [req][head][qmax*G][split][128]
    float* part_ml;           // [req][head][qmax*G][split][2]
    void* out;
    int out_dtype;
    int64_t out_stride;
    int32_t* status;
    // the merge's fused all-gather (ttkv_decode_paged_gather): n_peers > 0 stores every output row
    // also at the same offset of peer_out[p] (p != peer_rank) and counts one arrival per merge CTA
    // on every peer_sig[p]
    int n_peers, peer_rank;
    void* peer_out[TTKV_MAX_PEERS];
    unsigned long long* peer_sig[TTKV_MAX_PEERS];
    unsigned long long* peer_ticket;  // this rank's ticket word: the merge CTAs of a launch count
                                      // here; the last posts the launch's arrivals to every rank
};

struct Smem {
    float* dec;       // [r1][128]
    float* q;         // [QR][128]
    float* coef;      // [r1][TT]
    float* y;         // [TT][RS]
    float* p;         // [QR][TT]
    float* cosv;      // [TT][64]
    float* sinv;      // [TT][64]
    float* cs;        // [TT]
    float* krs;       // [TT]
    float* vrs;       // [TT]
    float* m;         // [QR]
    float* l;         // [QR]
    float* corr;      // [QR]
    uint32_t* kw;     // [TT][4]
    uint32_t* kpre;   // [TT][4]
    uint32_t* vw;     // [TT][4]
    uint32_t* vpre;   // [TT][4]
    int64_t* slot;    // [TT]
    uint8_t* krow;    // [TT][kpad]
    uint8_t* vrow;    // [TT][vpad]
    int kpad, vpad;
};

__host__ __device__ inline int pad4(int n) { return (n + 3) & ~3; }

__host__ __device__ inline size_t smem_bytes(int r1, int QR, int k_row, int v_row) {
    size_t f = size_t(r1) * 128 + size_t(QR) * 128 + size_t(r1) * TT + size_t(TT) * RS +
               size_t(QR) * TT + 2 * TT * 64 + 3 * TT + 3 * QR;
    size_t b = f * 4 + 4 * TT * 4 * 4 + 8 + TT * 8 + size_t(TT) * (pad4(k_row + 1) + pad4(v_row + 1));
    return (b + 15) & ~size_t(15);
}

__device__ inline Smem carve(unsigned char* base, int r1, int QR, int k_row, int v_row) {
    Smem s;
    float* f = reinterpret_cast<float*>(base);
    s.dec = f;  f += r1 * 128;
    s.q = f;    f += QR * 128;
    s.coef = f; f += r1 * TT;
    s.y = f;    f += TT * RS;
    s.p = f;    f += QR * TT;
    s.cosv = f; f += TT * 64;
    s.sinv = f; f += TT * 64;
    s.cs = f;   f += TT;
    s.krs = f;  f += TT;
    s.vrs = f;  f += TT;
    s.m = f;    f += QR;
    s.l = f;    f += QR;
    s.corr = f; f += QR;
    uint32_t* u = reinterpret_cast<uint32_t*>(f);
    s.kw = u;   u += TT * 4;
    s.kpre = u; u += TT * 4;
    s.vw = u;   u += TT * 4;
    s.vpre = u; u += TT * 4;
    // int64 slots need 8-byte alignment: every block above is a multiple of 4 floats except
    // the QR-sized ones, so round up here
    uintptr_t a = (reinterpret_cast<uintptr_t>(u) + 7) & ~uintptr_t(7);
    s.slot = reinterpret_cast<int64_t*>(a);
    unsigned char* b = reinterpret_cast<unsigned char*>(s.slot + TT);
    s.kpad = pad4(k_row + 1);
    s.vpad = pad4(v_row + 1);
    s.krow = b; b += TT * s.kpad;
    s.vrow = b;
    return s;
}

// Value of lane j in a staged packed row whose 4 bitmap words and their exclusive prefix
// popcounts are precomputed. A well-formed row has exactly `kmax` bits set; a malformed one
// (more bits) reads lanes past the kmax-th as zero instead of reading past the staged row.
__device__ __forceinline__ float staged_lane(const uint32_t* w, const uint32_t* pre,
                                             const uint8_t* stream, float ruler, int bits, int kmax,
                                             int j) {
    const int wi = j >> 5, l = j & 31;
    const uint32_t word = w[wi];
    if (!((word >> (31 - l)) & 1u)) return 0.f;
    const int rank = int(pre[wi]) + __popc(word & ~(0xffffffffu >> l));
    if (rank >= kmax) return 0.f;
    return float(code_at(stream, rank, bits) - (1 << (bits - 1))) * ruler;
}

template <int QR>
__device__ __forceinline__ void write_partial(const ReadParams& P, int r, int hl, int qrow0,
                                              int split, const float (&o)[QR], const Smem& S,
                                              int nrows) {
    const int tid = threadIdx.x;
    const int QG = P.qmax * P.G;
    #pragma unroll
    for (int i = 0; i < QR; ++i) {
        if (i < nrows) {
            const int64_t row = (int64_t(r) * P.n_heads + hl) * QG + qrow0 + i;
            P.part_o[(row * P.n_splits + split) * 128 + tid] = o[i];
            if (tid == 0) {
                P.part_ml[(row * P.n_splits + split) * 2 + 0] = S.m[i];
                P.part_ml[(row * P.n_splits + split) * 2 + 1] = S.l[i];
            }
        }
    }
}

// QB query tokens x G heads = QR query rows per CTA. MULTI: continuation (causal, q_start/q_len).
template <int G, int QB, bool MULTI>
__global__ void __launch_bounds__(NT) attn_split_kernel(const ReadParams P) {
    constexpr int QR = G * QB;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int tid = threadIdx.x;
    const int split = blockIdx.x;
    const int hl = blockIdx.y / P.n_qblk, qb = blockIdx.y % P.n_qblk;
    const int h = P.head_lo + hl;
    const int r = blockIdx.z;
    Smem S = carve(smem_raw, P.r1, QR, P.k_row, P.v_row);

    const int seq = P.seq_lens[r];
    const int qlen = MULTI ? P.q_len[r] : 1;
    const int qrow_first = MULTI ? P.q_start[r] : r;
    const int j0 = qb * QB;                               // first query of this block
    const int nq = min(QB, qlen - j0);                    // queries in this block
    const int nrows = max(nq, 0) * G;
    const int p0 = seq - qlen;                            // position of query 0

    float o[QR];
    #pragma unroll
    for (int i = 0; i < QR; ++i) o[i] = 0.f;
    if (tid < QR) { S.m[tid] = -INFINITY; S.l[tid] = 0.f; }

    // ---- validation: a refusal is recorded and the CTA contributes nothing
    const int di = P.dec_index[r];
    bool bad = false;
    if (nq <= 0) bad = true;                              // an empty query block: nothing to do
    if (!bad && seq > P.max_seq) { report(P.status, TTKV_STATUS_SEQ_BOUND); bad = true; }
    if (!bad && (MULTI && (qlen > seq || qlen < 0))) { report(P.status, TTKV_STATUS_QUERY); bad = true; }
    if (!bad && (di < 0 || di >= P.n_decoders)) { report(P.status, TTKV_STATUS_DECODER); bad = true; }
    const int blocks_needed = (seq + P.block_size - 1) / P.block_size;
    if (!bad && blocks_needed > P.bt_cols) { report(P.status, TTKV_STATUS_ROW_SHORT); bad = true; }
    int t_begin = split * P.chunk;
    int t_end = min(seq, t_begin + P.chunk);
    if (MULTI) t_end = min(t_end, p0 + j0 + nq);          // rows past the block's last query
    if (!bad && t_begin < t_end) {
        const int64_t n_blocks = P.n_slots / P.block_size;
        const int32_t* row = P.block_table + int64_t(r) * P.bt_stride;
        int local_bad = 0;
        for (int b = t_begin / P.block_size + tid; b <= (t_end - 1) / P.block_size; b += NT) {
            const int32_t blk = row[b];
            if (blk < 0 || blk >= n_blocks) local_bad = 1;
        }
        if (__syncthreads_or(local_bad)) {
            if (tid == 0) report(P.status, TTKV_STATUS_BLOCK_RANGE);
            bad = true;
        }
    }
    __syncthreads();
    if (bad || t_begin >= t_end) {
        write_partial<QR>(P, r, hl, j0 * G, split, o, S, nrows);
        return;
    }

    // ---- stage this head's decoder slice and the query rows
    const float* dec = P.decoders + int64_t(di) * P.dec_stride;
    for (int i = tid; i < P.r1 * 32; i += NT) {
        const int rr = i >> 5, c4 = i & 31;
        reinterpret_cast<float4*>(S.dec)[i] =
            reinterpret_cast<const float4*>(dec + int64_t(rr) * P.H * 128 + h * 128)[c4];
    }
    for (int i = tid; i < QR * 128; i += NT) {
        const int qr = i >> 7, lane = i & 127;
        const int jq = j0 + qr / G, g = qr % G;
        float v = 0.f;
        if (jq < qlen) {
            const int64_t e = int64_t(qrow_first + jq) * P.q_stride + int64_t(h * G + g) * 128 + lane;
            v = load_elt(P.q, P.q_dtype, e);
        }
        S.q[i] = v;
    }

    const int lg = tid & 15, tg = tid >> 4;               // lane group, token group
    const int32_t* brow = P.block_table + int64_t(r) * P.bt_stride;
    const int kfield = P.coeff_bytes + 2 + h * P.k_row;
    const int vfield = P.v_offset + h * P.v_row;

    for (int t0 = t_begin; t0 < t_end; t0 += TT) {
        __syncthreads();                                   // previous tile fully consumed
        // ---- gather: slots, rulers, residual / V rows, RoPE rows
        if (tid < TT) {
            const int t = t0 + tid;
            int64_t slot = -1;
            if (t < t_end) slot = int64_t(brow[t / P.block_size]) * P.block_size + t % P.block_size;
            S.slot[tid] = slot;
        }
        __syncthreads();
        if (tid < TT) {
            const int64_t slot = S.slot[tid];
            S.cs[tid] = slot >= 0 ? f16_at(P.cache + slot * P.row_bytes + P.coeff_bytes) : 0.f;
        }
        for (int i = tid; i < TT * P.k_row; i += NT) {
            const int t = i / P.k_row, b = i % P.k_row;
            const int64_t slot = S.slot[t];
            S.krow[t * S.kpad + b] = slot >= 0 ? P.cache[slot * P.row_bytes + kfield + b] : 0;
        }
        for (int i = tid; i < TT * P.v_row; i += NT) {
            const int t = i / P.v_row, b = i % P.v_row;
            const int64_t slot = S.slot[t];
            S.vrow[t * S.vpad + b] = slot >= 0 ? P.cache[slot * P.row_bytes + vfield + b] : 0;
        }
        for (int i = tid; i < TT * 64; i += NT) {
            const int t = i >> 6, c = i & 63;
            const int pos = min(t0 + t, int(P.table_rows - 1));
            S.cosv[i] = load_elt(P.table, P.table_dtype, int64_t(pos) * 128 + c);
            S.sinv[i] = load_elt(P.table, P.table_dtype, int64_t(pos) * 128 + 64 + c);
        }
        __syncthreads();
        for (int i = tid; i < P.r1 * TT; i += NT) {
            const int rr = i / TT, t = i % TT;
            const int64_t slot = S.slot[t];
            const float cq = slot >= 0 ? float(int8_t(P.cache[slot * P.row_bytes + rr])) : 0.f;
            S.coef[rr * TT + t] = cq * S.cs[t];           // g = cq * cs, exact in fp32
        }
        if (tid < TT) {
            const uint8_t* kr = S.krow + tid * S.kpad;
            const uint8_t* vr = S.vrow + tid * S.vpad;
            uint32_t kp = 0, vp = 0;
            #pragma unroll
            for (int w = 0; w < 4; ++w) {
                const uint32_t kw = bitmap_word(kr, w), vw = bitmap_word(vr, w);
                S.kw[tid * 4 + w] = kw; S.kpre[tid * 4 + w] = kp; kp += __popc(kw);
                S.vw[tid * 4 + w] = vw; S.vpre[tid * 4 + w] = vp; vp += __popc(vw);
            }
            S.krs[tid] = f16_at(kr + 16 + P.k_pb);
            S.vrs[tid] = f16_at(vr + 16 + P.v_pb);
        }
        __syncthreads();

        // ---- rebuild + patch + rotate: thread owns tokens 4tg..4tg+3, lanes 4lg.. and 64+4lg..
        {
            float acc[4][8];
            #pragma unroll
            for (int t = 0; t < 4; ++t)
                #pragma unroll
                for (int c = 0; c < 8; ++c) acc[t][c] = 0.f;
            for (int rr = 0; rr < P.r1; ++rr) {
                const float4 dl = *reinterpret_cast<const float4*>(S.dec + rr * 128 + 4 * lg);
                const float4 dh = *reinterpret_cast<const float4*>(S.dec + rr * 128 + 64 + 4 * lg);
                const float4 cv = *reinterpret_cast<const float4*>(S.coef + rr * TT + 4 * tg);
                const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
                const float dd[8] = {dl.x, dl.y, dl.z, dl.w, dh.x, dh.y, dh.z, dh.w};
                #pragma unroll
                for (int t = 0; t < 4; ++t)
                    #pragma unroll
                    for (int c = 0; c < 8; ++c) acc[t][c] = fmaf(cc[t], dd[c], acc[t][c]);
            }
            #pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int tt = 4 * tg + t;
                const uint8_t* stream = S.krow + tt * S.kpad + 16;
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int jl = 4 * lg + c, jh = 64 + 4 * lg + c;
                    const float klo = acc[t][c] + staged_lane(S.kw + tt * 4, S.kpre + tt * 4, stream,
                                                              S.krs[tt], P.res_bits, P.res_k, jl);
                    const float khi = acc[t][4 + c] + staged_lane(S.kw + tt * 4, S.kpre + tt * 4, stream,
                                                                  S.krs[tt], P.res_bits, P.res_k, jh);
                    const float cz = S.cosv[tt * 64 + jl], sz = S.sinv[tt * 64 + jl];
                    S.y[tt * RS + jl] = klo * cz - khi * sz;
                    S.y[tt * RS + jh] = khi * cz + klo * sz;
                }
            }
        }
        __syncthreads();

        // ---- scores: one (query row, token) pair per thread-iteration
        for (int i = tid; i < QR * TT; i += NT) {
            const int qr = i / TT, t = i % TT;
            const int jq = j0 + qr / G;
            const int tabs = t0 + t;
            float s = -INFINITY;
            const bool live = tabs < t_end && qr < nrows && (!MULTI || tabs <= p0 + jq);
            if (live) {
                const float4* yr = reinterpret_cast<const float4*>(S.y + t * RS);
                const float4* qv = reinterpret_cast<const float4*>(S.q + qr * 128);
                float a = 0.f;
                #pragma unroll 8
                for (int c = 0; c < 32; ++c) {
                    const float4 x = yr[c], w = qv[c];
                    a = fmaf(x.x, w.x, a); a = fmaf(x.y, w.y, a);
                    a = fmaf(x.z, w.z, a); a = fmaf(x.w, w.w, a);
                }
                s = a * P.scale;
            }
            S.p[qr * TT + t] = s;
        }
        __syncthreads();

        // ---- online softmax: one warp per query row
        for (int qr = tid >> 5; qr < QR; qr += NT / 32) {
            const int lane = tid & 31;
            const float s = S.p[qr * TT + lane];
            float mx = s;
            #pragma unroll
            for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_old = S.m[qr];
            const float m_new = fmaxf(m_old, mx);
            float pe = 0.f, corr = 1.f;
            if (m_new != -INFINITY) {
                pe = (s == -INFINITY) ? 0.f : expf(s - m_new);
                corr = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
            }
            float sum = pe;
            #pragma unroll
            for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            S.p[qr * TT + lane] = pe;
            __syncwarp();
            if (lane == 0) {
                S.l[qr] = S.l[qr] * corr + sum;
                S.m[qr] = m_new;
                S.corr[qr] = corr;
            }
        }
        __syncthreads();

        // ---- readout: thread = lane
        {
            #pragma unroll
            for (int i = 0; i < QR; ++i) o[i] *= S.corr[i];
            const int ntok = min(TT, t_end - t0);
            for (int t = 0; t < ntok; ++t) {
                const float v = staged_lane(S.vw + t * 4, S.vpre + t * 4, S.vrow + t * S.vpad + 16,
                                            S.vrs[t], P.v_bits, P.v_lanes, tid);
                #pragma unroll
                for (int i = 0; i < QR; ++i) o[i] = fmaf(S.p[i * TT + t], v, o[i]);
            }
        }
    }
    __syncthreads();
    write_partial<QR>(P, r, hl, j0 * G, split, o, S, nrows);
}

// Combine the splits of one (request, KV head, query row): thread = lane.
__global__ void __launch_bounds__(128) merge_kernel(const ReadParams P) {
    const int qr = blockIdx.x, hl = blockIdx.y, r = blockIdx.z, lane = threadIdx.x;
    const int jq = qr / P.G, g = qr % P.G;
    const int qlen = P.q_len ? P.q_len[r] : 1;
    if (jq >= qlen) return;
    const int QG = P.qmax * P.G;
    const int64_t row = (int64_t(r) * P.n_heads + hl) * QG + qr;
    float M = -INFINITY;
    for (int s = 0; s < P.n_splits; ++s) M = fmaxf(M, P.part_ml[(row * P.n_splits + s) * 2]);
    float acc = 0.f, den = 0.f;
    if (M != -INFINITY) {
        for (int s = 0; s < P.n_splits; ++s) {
            const float ms = P.part_ml[(row * P.n_splits + s) * 2];
            if (ms == -INFINITY) continue;
            const float w = expf(ms - M);
            acc = fmaf(w, P.part_o[(row * P.n_splits + s) * 128 + lane], acc);
            den = fmaf(w, P.part_ml[(row * P.n_splits + s) * 2 + 1], den);
        }
    }
    const float v = den > 0.f ? acc / den : 0.f;
    const int qrow = (P.q_start ? P.q_start[r] : r) + jq;
    const int head_q = (P.head_lo + hl) * P.G + g;
    store_elt(P.out, P.out_dtype, int64_t(qrow) * P.out_stride + int64_t(head_q) * 128 + lane, v);
}

#include "ttkv_decode_tc.cuh"
#include "ttkv_cont_tc.cuh"

// ------------------------------------------------------------------ host side
int qblock_for(int G, bool multi) {
    if (!multi) return 1;
    return G <= 3 ? 16 : (G <= 6 ? 8 : 4);               // G*QB <= 48 query rows per CTA
}

struct Plan {
    int qb, n_qblk, n_splits, chunk;
    size_t part_o_bytes, part_ml_bytes, smem;
    long long n_part_slots;
};

Plan make_plan(const ttkv_layout_t* lay, int n_reqs, int HQ, int max_q, int max_seq,
               int n_heads, bool multi) {
    Plan pl{};
    const int G = HQ / lay->H;
    pl.qb = qblock_for(G, multi);
    const int qmax = multi ? max(max_q, 1) : 1;
    pl.n_qblk = (qmax + pl.qb - 1) / pl.qb;
    const int base = max(1, n_reqs * n_heads * pl.n_qblk);
    const int max_tiles = max(1, (max_seq + TT - 1) / TT);
    int want = (2 * 148 + base - 1) / base;                // about two CTAs per SM
    want = max(1, min(want, max_tiles));
    const int tiles_per_split = (max_tiles + want - 1) / want;
    pl.chunk = tiles_per_split * TT;
    pl.n_splits = max(1, (max_seq + pl.chunk - 1) / pl.chunk);
    const size_t rows = size_t(n_reqs) * n_heads * qmax * G;
    pl.part_o_bytes = rows * pl.n_splits * 128 * sizeof(float);
    pl.part_ml_bytes = rows * pl.n_splits * 2 * sizeof(float);
    pl.smem = smem_bytes(lay->r1, G * pl.qb, lay->k_row_bytes, lay->v_row_bytes);
    return pl;
}

int sm_count() {
    static int cached = 0;
    if (cached) return cached;
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
        cached = n;
    else
        cudaGetLastError();                                   // clear; plan for a full B200
    return cached ? cached : 148;
}

// Whether the tensor-core decode serves this layout (the fp32 kernel serves the rest).
bool tc_serves(const ttkv_layout_t* lay, int HQ) {
    const int G = HQ / lay->H;
    // code windows hold 8 codes in 32 bits: widths up to 4 bits
    return lay->d == 128 && lay->qbits == 8 && G >= 1 && G <= kMaxG && lay->r1 <= tc::MAX_R1 &&
           lay->res_bits <= 4 && lay->v_bits <= 4 && lay->res_k <= 128 && lay->v_lanes <= 128 &&
           tc::tc_geom(lay, G).smem > 0;
}

// The tensor-core decode's grid: one resident CTA per SM (fewer only when the batch has fewer
// units), each taking an equal share of the (request, KV head, tile) units; the grid does not
// depend on max_seq beyond that, so a graph captured with a bound replays any batch within it. The
// device cuts the shares into virtual shares when a segment would outgrow the cached block-table
// slice. Partials: one slot per (virtual share, pair) that can meet, share index + pair index, so
// the workspace holds (CTAs x the most virtual shares max_seq allows) + pairs slots. block_size 1
// needs the most shares, so a workspace sized for it covers every block size.
Plan make_plan_tc(const ttkv_layout_t* lay, int n_reqs, int HQ, int max_seq, int n_heads, int block_size) {
    Plan pl{};
    const int G = HQ / lay->H;
    pl.qb = 1;
    pl.n_qblk = 1;
    const long long tiles = std::max(1, (max_seq + tc::TM - 1) / tc::TM);
    const long long pairs = std::max(1LL, (long long)n_reqs * n_heads);
    const long long units = pairs * tiles;
    const long long n = std::min<long long>(sm_count(), units);
    pl.n_splits = int(n);
    pl.chunk = 0;
    const size_t slots = size_t(n * tc::virtual_shares(units, n, block_size) + pairs);
    pl.n_part_slots = (long long)slots;
    pl.part_o_bytes = slots * G * 128 * sizeof(float);
    pl.part_ml_bytes = slots * G * 2 * sizeof(float);
    pl.smem = size_t(tc::tc_geom(lay, G).smem);
    return pl;
}

// Continuation chunks on the tensor-core decode: the (query, query head) rows of a request's
// chunk, query-major, in blocks of the decode's 8 rows; each block is one request of a decode
// launch with G = 8, so each stored tile is rebuilt once per 8 rows (8 / G queries) instead of
// once per query.
constexpr int kContRows = kMaxG;

struct ContPlan {
    int nqb, n_v;            // blocks per request, blocks in all
    Plan pl;                 // the decode's plan over the n_v blocks
    size_t arrays_off;       // six int32 [n_v] arrays (block rows, request, first query row, row
    size_t bytes;            // count, first query's position, first row) after the partials
};

ContPlan make_cont_plan(const ttkv_layout_t* lay, int n_reqs, int HQ, int max_q, int max_seq,
                        int n_heads, int block_size) {
    ContPlan c{};
    const int G = HQ / lay->H;
    c.nqb = int((int64_t(max_q) * G + kContRows - 1) / kContRows);
    c.n_v = n_reqs * c.nqb;
    c.pl = make_plan_tc(lay, c.n_v, lay->H * kContRows, max_seq, n_heads, block_size);
    c.arrays_off = (c.pl.part_o_bytes + c.pl.part_ml_bytes + 255) & ~size_t(255);
    c.bytes = c.arrays_off + size_t(6) * c.n_v * sizeof(int32_t);
    return c;
}

int check_common(const ttkv_layout_t* lay, const ttkv_cache_t* cache, const ttkv_batch_t* batch,
                 const ttkv_rope_t* rope, int HQ, int head_lo, int head_hi) {
    if (!lay || !cache || !batch || !rope) return fail(TTKV_ERR_ARG, "null layout/cache/batch/rope");
    if (lay->d != kHeadDim) return fail(TTKV_ERR_UNSUPPORTED, "head dim %d: the kernels serve d=128", lay->d);
    if (lay->qbits != 8) return fail(TTKV_ERR_UNSUPPORTED, "qbits=%d: coefficients are int8", lay->qbits);
    if (lay->r1 < 1 || lay->r1 > kMaxRank)
        return fail(TTKV_ERR_UNSUPPORTED, "r1=%d outside 1..%d", lay->r1, kMaxRank);
    if (lay->res_k < 1) return fail(TTKV_ERR_UNSUPPORTED, "res_k=0 (no residual) is not served");
    if (HQ < lay->H || HQ % lay->H)
        return fail(TTKV_ERR_ARG, "HQ=%d is not a multiple of H=%d", HQ, lay->H);
    if (HQ / lay->H > kMaxG) return fail(TTKV_ERR_UNSUPPORTED, "GQA group %d > %d", HQ / lay->H, kMaxG);
    if (head_lo < 0 || head_hi > lay->H || head_lo >= head_hi)
        return fail(TTKV_ERR_ARG, "head range [%d, %d) outside [0, %d)", head_lo, head_hi, lay->H);
    if (!cache->base || cache->block_size < 1 || cache->n_slots < 0 || cache->row_bytes < lay->blob_bytes)
        return fail(TTKV_ERR_ARG, "cache rows are %lld bytes, the layout needs %d",
                    (long long)cache->row_bytes, lay->blob_bytes);
    if (!batch->block_table || !batch->seq_lens || !batch->decoders || !batch->dec_index || batch->n_reqs < 0)
        return fail(TTKV_ERR_ARG, "batch has a null pointer");
    if (batch->dec_stride < int64_t(lay->r1) * lay->H * 128)
        return fail(TTKV_ERR_ARG, "decoder stride %lld < r1*H*d", (long long)batch->dec_stride);
    if ((reinterpret_cast<uintptr_t>(batch->decoders) & 15) || (batch->dec_stride & 3))
        return fail(TTKV_ERR_ALIGN, "decoders must be 16-byte aligned with a stride of 4 floats");
    if (batch->dec_image) {
        const size_t img = tc_serves(lay, HQ) ? tc::image_bytes(lay) : 0;
        if (img && ((reinterpret_cast<uintptr_t>(batch->dec_image) & 15) || (batch->image_stride & 15) ||
                    batch->image_stride < int64_t(img) || !batch->dec_scales))
            return fail(TTKV_ERR_ALIGN, "decoder images must be 16-byte aligned, %zu bytes apart at least, "
                        "with their scales", img);
    }
    if (!rope->table || rope->rows < 1) return fail(TTKV_ERR_ARG, "RoPE table missing");
    if (rope->dtype < TTKV_F32 || rope->dtype > TTKV_BF16) return fail(TTKV_ERR_ARG, "RoPE dtype");
    return TTKV_OK;
}

ReadParams base_params(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                       const ttkv_batch_t* batch, const ttkv_rope_t* rope) {
    ReadParams P{};
    P.H = lay->H; P.r1 = lay->r1; P.res_k = lay->res_k; P.res_bits = lay->res_bits;
    P.v_lanes = lay->v_lanes; P.v_bits = lay->v_bits;
    P.coeff_bytes = lay->coeff_bytes; P.k_row = lay->k_row_bytes; P.v_row = lay->v_row_bytes;
    P.v_offset = lay->v_offset;
    P.k_pb = packed_row_bytes(lay->res_k, lay->res_bits);
    P.v_pb = packed_row_bytes(lay->v_lanes, lay->v_bits);
    P.cache = cache->base; P.n_slots = cache->n_slots; P.row_bytes = cache->row_bytes;
    P.block_size = cache->block_size;
    P.block_table = batch->block_table; P.bt_stride = batch->bt_stride; P.bt_cols = batch->bt_cols;
    P.seq_lens = batch->seq_lens; P.decoders = batch->decoders; P.dec_stride = batch->dec_stride;
    P.dec_index = batch->dec_index; P.n_decoders = batch->n_decoders;
    P.dec_image = static_cast<const unsigned char*>(batch->dec_image);
    P.image_stride = batch->image_stride; P.dec_scales = batch->dec_scales;
    P.table = rope->table; P.table_dtype = rope->dtype; P.table_rows = rope->rows;
    return P;
}

template <int G, int QB, bool MULTI>
int launch_g(const ReadParams& P, const Plan& pl, int n_reqs, cudaStream_t st) {
    auto k = attn_split_kernel<G, QB, MULTI>;
    if (int e = raise_smem_limit(reinterpret_cast<const void*>(k), "attn_split_kernel")) return e;
    dim3 grid(pl.n_splits, P.n_heads * pl.n_qblk, n_reqs);
    k<<<grid, NT, pl.smem, st>>>(P);
    if (int e = check_launch("attn_split_kernel")) return e;
    dim3 mg(P.qmax * P.G, P.n_heads, n_reqs);
    merge_kernel<<<mg, 128, 0, st>>>(P);
    return check_launch("merge_kernel");
}

// The TMA map of a tensor-core decode launch (the RoPE table, only when its rows are staged).
bool tc_maps(tc::TcMaps* M, const tc::TcGeom& T, const ReadParams& P) {
    memset(M, 0, sizeof(*M));
    if (!T.rope_smem) return true;
    return encode_2d(&M->rope, CU_TENSOR_MAP_DATA_TYPE_UINT16, P.table, 128, uint64_t(P.table_rows), 256, 64, 128, 128);
}

template <int G>
int launch_tc_g(const ReadParams& P, const tc::TcGeom& T, const tc::TcMaps& maps, const Plan& pl, int n_reqs,
                cudaStream_t st) {
    auto k = P.table_dtype == TTKV_BF16 ? tc::decode_tc_kernel<G, true> : tc::decode_tc_kernel<G, false>;
    if (int e = raise_smem_limit(reinterpret_cast<const void*>(k), "decode_tc_kernel")) return e;
    // both launches may start while the kernel before them runs (programmatic dependent launch):
    // the decode waits for the step's write before its first cache read, the merge for the decode
    // before its first partial
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(P.n_ctas);
    cfg.blockDim = dim3(tc::NTHR);
    cfg.dynamicSmemBytes = T.smem;
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, P, T, maps);
    if (e != cudaSuccess) return fail(TTKV_ERR_CUDA, "decode_tc_kernel: %s", cudaGetErrorString(e));
    cfg.gridDim = dim3(P.G, P.n_heads, n_reqs);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = 0;
    e = cudaLaunchKernelEx(&cfg, tc::merge_sk_kernel, P);
    if (e != cudaSuccess) return fail(TTKV_ERR_CUDA, "merge_sk_kernel: %s", cudaGetErrorString(e));
    return TTKV_OK;
}

int launch_tc(const ReadParams& P, const tc::TcGeom& T, const tc::TcMaps& maps, const Plan& pl, int n_reqs,
              cudaStream_t st) {
    switch (P.G) {
        case 1: return launch_tc_g<1>(P, T, maps, pl, n_reqs, st);
        case 2: return launch_tc_g<2>(P, T, maps, pl, n_reqs, st);
        case 3: return launch_tc_g<3>(P, T, maps, pl, n_reqs, st);
        case 4: return launch_tc_g<4>(P, T, maps, pl, n_reqs, st);
        case 5: return launch_tc_g<5>(P, T, maps, pl, n_reqs, st);
        case 6: return launch_tc_g<6>(P, T, maps, pl, n_reqs, st);
        case 7: return launch_tc_g<7>(P, T, maps, pl, n_reqs, st);
        case 8: return launch_tc_g<8>(P, T, maps, pl, n_reqs, st);
    }
    return fail(TTKV_ERR_UNSUPPORTED, "GQA group %d", P.G);
}

// Whether cont_tc_kernel serves a continuation call: the tensor-core layouts whose coefficient
// block fits one 128-byte row (r1 <= 126), a 16-bit query (it is an MMA operand as is, read as
// 16-byte rows), the decoders' operand images, and 16-byte aligned slot rows and RoPE rows.
bool ct_serves(const ttkv_layout_t* lay, int HQ, const ttkv_batch_t* batch, const ttkv_cache_t* cache,
               const ttkv_rope_t* rope, const void* q, int32_t q_dtype, int64_t q_stride) {
    return tc_serves(lay, HQ) && ct::ct_geom(lay, HQ / lay->H, cache->block_size).smem > 0 &&
           batch->dec_image && batch->dec_scales && batch->n_reqs <= 65535 &&
           (q_dtype == TTKV_F16 || q_dtype == TTKV_BF16) &&
           (reinterpret_cast<uintptr_t>(q) & 15) == 0 && (q_stride & 7) == 0 && rope->dtype != TTKV_F32 &&
           (reinterpret_cast<uintptr_t>(rope->table) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(cache->base) & 15) == 0 && (cache->row_bytes & 15) == 0;
}

int launch_ct(const ReadParams& P, const ct::CtGeom& T, int max_q_len, int n_reqs, cudaStream_t st) {
    auto k = ct::cont_tc_kernel;
    if (int e = raise_smem_limit(reinterpret_cast<const void*>(k), "cont_tc_kernel")) return e;
    // may start while the step's write runs (programmatic dependent launch): the kernel waits for
    // it before its first read
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned((int64_t(max_q_len) * P.G + tc::TM - 1) / tc::TM), P.n_heads, n_reqs);
    cfg.blockDim = dim3(ct::NTHR);
    cfg.dynamicSmemBytes = T.smem;
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k, P, T);
    if (e != cudaSuccess) return fail(TTKV_ERR_CUDA, "cont_tc_kernel: %s", cudaGetErrorString(e));
    return TTKV_OK;
}

template <bool MULTI>
int launch(const ReadParams& P, const Plan& pl, int n_reqs, cudaStream_t st) {
    switch (P.G) {
        case 1: return launch_g<1, (MULTI ? 16 : 1), MULTI>(P, pl, n_reqs, st);
        case 2: return launch_g<2, (MULTI ? 16 : 1), MULTI>(P, pl, n_reqs, st);
        case 3: return launch_g<3, (MULTI ? 16 : 1), MULTI>(P, pl, n_reqs, st);
        case 4: return launch_g<4, (MULTI ? 8 : 1), MULTI>(P, pl, n_reqs, st);
        case 5: return launch_g<5, (MULTI ? 8 : 1), MULTI>(P, pl, n_reqs, st);
        case 6: return launch_g<6, (MULTI ? 8 : 1), MULTI>(P, pl, n_reqs, st);
        case 7: return launch_g<7, (MULTI ? 4 : 1), MULTI>(P, pl, n_reqs, st);
        case 8: return launch_g<8, (MULTI ? 4 : 1), MULTI>(P, pl, n_reqs, st);
    }
    return fail(TTKV_ERR_UNSUPPORTED, "GQA group %d", P.G);
}

// The gathered decode's wait (ttkv_peer_wait): this rank's signal word must reach the arrivals
// waited for so far plus this step's, every rank's merge CTAs of this step having stored their rows
// here first (each fenced its stores system-wide before its arrival). One thread polls with an
// acquire load; the wait is bounded, and the count waited for advances either way.
__global__ void peer_wait_kernel(const unsigned long long* sig, unsigned long long* waited,
                                 unsigned long long arrivals, int32_t* status) {
    if (threadIdx.x != 0) return;
    const unsigned long long target = *waited + arrivals;
    const long long t0 = clock64();
    bool ok = true;
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(sig) : "memory");
        if (v >= target) break;
        if (clock64() - t0 > kWaitCycles) { ok = false; break; }
        __nanosleep(128);
    }
    *waited = target;
    if (!ok) report(status, TTKV_STATUS_TIMEOUT);
    __threadfence_system();
}

}  // namespace
}  // namespace ttkv

using namespace ttkv;

namespace {
// Scratch of a decode for caches of `block_size` tokens per block (1 covers every block size).
size_t decode_workspace(const ttkv_layout_t* lay, int32_t n_reqs, int32_t HQ, int32_t max_seq_len,
                        int32_t head_lo, int32_t head_hi, int block_size) {
    if (!lay || lay->H < 1 || HQ < lay->H || head_hi <= head_lo) return 0;
    const Plan pl = make_plan(lay, n_reqs, HQ, 1, max_seq_len, head_hi - head_lo, false);
    size_t need = pl.part_o_bytes + pl.part_ml_bytes;
    if (tc_serves(lay, HQ)) {
        const Plan pt = make_plan_tc(lay, n_reqs, HQ, max_seq_len, head_hi - head_lo, block_size);
        need = std::max(need, pt.part_o_bytes + pt.part_ml_bytes);
    }
    return need;
}
}  // namespace

extern "C" size_t ttkv_decode_workspace_bytes(const ttkv_layout_t* lay, int32_t n_reqs, int32_t HQ,
                                              int32_t max_seq_len, int32_t head_lo, int32_t head_hi) {
    return decode_workspace(lay, n_reqs, HQ, max_seq_len, head_lo, head_hi, 1);
}

extern "C" size_t ttkv_prefill_workspace_bytes(const ttkv_layout_t* lay, int32_t n_reqs, int32_t HQ,
                                               int32_t max_q_len, int32_t max_seq_len,
                                               int32_t head_lo, int32_t head_hi) {
    if (!lay || lay->H < 1 || HQ < lay->H || head_hi <= head_lo) return 0;
    const Plan pl = make_plan(lay, n_reqs, HQ, max_q_len, max_seq_len, head_hi - head_lo, true);
    size_t need = pl.part_o_bytes + pl.part_ml_bytes;
    if (max_q_len >= 1 && tc_serves(lay, lay->H * kContRows))            // sized for blocks of 16 tokens
        need = std::max(need, make_cont_plan(lay, n_reqs, HQ, max_q_len, max_seq_len, head_hi - head_lo,
                                             16).bytes);
    return need;
}

// The host-side refusals every read makes before it looks at its scratch.
static int check_read_args(bool multi, const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                           const ttkv_batch_t* batch, const ttkv_rope_t* rope, const int32_t* q_start,
                           const int32_t* q_len, const void* q, int32_t q_dtype, int64_t q_stride,
                           int32_t HQ, int32_t head_lo, int32_t head_hi, const void* out,
                           int32_t out_dtype, int64_t out_stride, int32_t max_q_len, int32_t max_seq_len) {
    if (int e = check_common(lay, cache, batch, rope, HQ, head_lo, head_hi)) return e;
    if (!q || !out) return fail(TTKV_ERR_ARG, "q/out null");
    if (q_dtype < TTKV_F32 || q_dtype > TTKV_BF16 || out_dtype < TTKV_F32 || out_dtype > TTKV_BF16)
        return fail(TTKV_ERR_ARG, "q/out dtype");
    if (q_stride < int64_t(HQ) * 128 || out_stride < int64_t(HQ) * 128)
        return fail(TTKV_ERR_ARG, "q/out stride below HQ*d");
    if (multi && (!q_start || !q_len)) return fail(TTKV_ERR_ARG, "q_start/q_len null");
    if (max_seq_len < 0 || (multi && max_q_len < 1)) return fail(TTKV_ERR_ARG, "max lengths");
    if (max_seq_len > rope->rows)
        return fail(TTKV_ERR_ARG, "position %d is past the model's cos_sin_cache, which holds %lld rows",
                    max_seq_len - 1, (long long)rope->rows);
    return TTKV_OK;
}

static int read_entry(bool multi, const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                      const ttkv_batch_t* batch, const ttkv_rope_t* rope, const int32_t* q_start,
                      const int32_t* q_len, const void* q, int32_t q_dtype, int64_t q_stride,
                      int32_t HQ, float scale, int32_t head_lo, int32_t head_hi, void* out,
                      int32_t out_dtype, int64_t out_stride, int32_t max_q_len, int32_t max_seq_len,
                      void* workspace, size_t ws_bytes, int32_t* status, void* stream,
                      const ttkv_peers_t* peers = nullptr) {
    if (int e = check_read_args(multi, lay, cache, batch, rope, q_start, q_len, q, q_dtype, q_stride, HQ,
                                head_lo, head_hi, out, out_dtype, out_stride, max_q_len, max_seq_len))
        return e;
    if (batch->n_reqs == 0 || max_seq_len == 0) return TTKV_OK;
    const int n_heads = head_hi - head_lo;
    // the tensor-core kernel divides token indices by the block size as a 32-bit multiply-high and
    // stages slots with TMA maps (when the driver cannot encode them the fp32 kernel serves)
    bool use_tc = !multi && tc_serves(lay, HQ) && rope->dtype != TTKV_F32 &&
                  (reinterpret_cast<uintptr_t>(rope->table) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(cache->base) & 15) == 0 && (cache->row_bytes & 15) == 0 &&
                  (int64_t(max_seq_len) + 256) * cache->block_size < (int64_t(1) << 30);
    ReadParams P = base_params(lay, cache, batch, rope);
    tc::TcGeom T{};
    tc::TcMaps maps;
    if (use_tc) {
        T = tc::tc_geom(lay, HQ / lay->H);
        use_tc = tc_maps(&maps, T, P);
    }
    if (peers) {
        if (!use_tc)
            return fail(TTKV_ERR_UNSUPPORTED, "the gathered decode needs the tensor-core decode (r1=%d)", lay->r1);
        P.n_peers = peers->world;
        P.peer_rank = peers->rank;
        P.peer_ticket = peers->ticket;
        for (int i = 0; i < peers->world; ++i) { P.peer_out[i] = peers->out[i]; P.peer_sig[i] = peers->signal[i]; }
    }
    const int Gq = HQ / lay->H;
    // continuation chunks: blocks of up to 128 (query, head) rows with every product on the tensor
    // cores, when cont_tc_kernel serves the call (no scratch)
    if (multi && ct_serves(lay, HQ, batch, cache, rope, q, q_dtype, q_stride)) {
        P.q = q; P.q_dtype = q_dtype; P.q_stride = q_stride; P.HQ = HQ; P.G = Gq;
        P.q_start = q_start; P.q_len = q_len;
        P.scale = scale; P.head_lo = head_lo; P.n_heads = n_heads;
        P.n_reqs = batch->n_reqs; P.max_seq = max_seq_len;
        P.out = out; P.out_dtype = out_dtype; P.out_stride = out_stride; P.status = status;
        return launch_ct(P, ct::ct_geom(lay, Gq, cache->block_size), max_q_len, batch->n_reqs,
                         reinterpret_cast<cudaStream_t>(stream));
    }
    // else blocks of 8 (query, head) rows on the tensor-core decode when it serves the layout at 8
    // rows and the workspace holds its plan (else the fp32 kernel below)
    if (multi && tc_serves(lay, lay->H * kContRows) && rope->dtype != TTKV_F32 &&
        (reinterpret_cast<uintptr_t>(rope->table) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(cache->base) & 15) == 0 && (cache->row_bytes & 15) == 0 &&
        (int64_t(max_seq_len) + 256) * cache->block_size < (int64_t(1) << 30)) {
        const ContPlan c = make_cont_plan(lay, batch->n_reqs, HQ, max_q_len, max_seq_len, n_heads,
                                          cache->block_size);
        tc::TcGeom TC = tc::tc_geom(lay, kContRows);
        tc::TcMaps mc;
        // the merge's grid holds one z-index per block (at most 65535)
        if (workspace && ws_bytes >= c.bytes && c.n_v <= 65535 && TC.smem > 0 && tc_maps(&mc, TC, P)) {
            int32_t* arr = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + c.arrays_off);
            int32_t *v_seq = arr, *v_req = arr + c.n_v, *v_qrow = arr + 2 * c.n_v;
            int32_t *v_nq = arr + 3 * c.n_v, *v_pos = arr + 4 * c.n_v, *v_f0 = arr + 5 * c.n_v;
            P.q = q; P.q_dtype = q_dtype; P.q_stride = q_stride; P.G = kContRows; P.HQ = lay->H * P.G;
            P.g_real = Gq; P.scale = scale; P.head_lo = head_lo; P.n_heads = n_heads;
            P.qmax = 1; P.n_qblk = 1; P.n_splits = c.pl.n_splits; P.chunk = 0;
            P.n_reqs = c.n_v; P.seq_lens = v_seq;
            P.v_req = v_req; P.v_qrow = v_qrow; P.v_nq = v_nq; P.v_pos = v_pos; P.v_f0 = v_f0;
            P.n_ctas = c.pl.n_splits; P.max_seq = max_seq_len; P.n_part_slots = c.pl.n_part_slots;
            P.part_o = reinterpret_cast<float*>(workspace);
            P.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + c.pl.part_o_bytes);
            P.out = out; P.out_dtype = out_dtype; P.out_stride = out_stride; P.status = status;
            cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
            tc::cont_blocks_kernel<<<(c.n_v + 255) / 256, 256, 0, st>>>(
                batch->seq_lens, q_start, q_len, batch->n_reqs, c.nqb, Gq, kContRows, v_seq, v_req,
                v_qrow, v_nq, v_pos, v_f0, status);
            if (int e = check_launch("cont_blocks_kernel")) return e;
            return launch_tc(P, TC, mc, c.pl, c.n_v, st);
        }
    }
    const Plan pl = use_tc ? make_plan_tc(lay, batch->n_reqs, HQ, max_seq_len, n_heads, cache->block_size)
                           : make_plan(lay, batch->n_reqs, HQ, max_q_len, max_seq_len, n_heads, multi);
    if (pl.smem > 227 * 1024) return fail(TTKV_ERR_UNSUPPORTED, "r1=%d needs %zu B of shared memory", lay->r1, pl.smem);
    if (!workspace || ws_bytes < pl.part_o_bytes + pl.part_ml_bytes)
        return fail(TTKV_ERR_WORKSPACE, "workspace %zu < %zu bytes", ws_bytes, pl.part_o_bytes + pl.part_ml_bytes);
    P.q = q; P.q_dtype = q_dtype; P.q_stride = q_stride; P.HQ = HQ; P.G = HQ / lay->H;
    P.q_start = multi ? q_start : nullptr; P.q_len = multi ? q_len : nullptr;
    P.scale = scale; P.head_lo = head_lo; P.n_heads = n_heads;
    P.qmax = multi ? max_q_len : 1; P.n_qblk = pl.n_qblk; P.n_splits = pl.n_splits; P.chunk = pl.chunk;
    P.n_reqs = batch->n_reqs; P.n_ctas = use_tc ? pl.n_splits : 0;
    P.max_seq = max_seq_len; P.n_part_slots = pl.n_part_slots;
    P.part_o = reinterpret_cast<float*>(workspace);
    P.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.part_o_bytes);
    P.out = out; P.out_dtype = out_dtype; P.out_stride = out_stride; P.status = status;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (use_tc) return launch_tc(P, T, maps, pl, batch->n_reqs, st);
    return multi ? launch<true>(P, pl, batch->n_reqs, st) : launch<false>(P, pl, batch->n_reqs, st);
}

extern "C" int ttkv_decode_paged(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                                 const ttkv_batch_t* batch, const ttkv_rope_t* rope, const void* q,
                                 int32_t q_dtype, int64_t q_stride, int32_t HQ, float scale,
                                 int32_t head_lo, int32_t head_hi, void* out, int32_t out_dtype,
                                 int64_t out_stride, int32_t max_seq_len, void* workspace,
                                 size_t workspace_bytes, int32_t* status, void* stream) {
    return read_entry(false, lay, cache, batch, rope, nullptr, nullptr, q, q_dtype, q_stride, HQ, scale,
                      head_lo, head_hi, out, out_dtype, out_stride, 1, max_seq_len, workspace,
                      workspace_bytes, status, stream);
}

extern "C" size_t ttkv_decoder_image_bytes(const ttkv_layout_t* lay) {
    if (!lay || lay->d != kHeadDim || lay->r1 < 1 || lay->r1 > tc::MAX_R1) return 0;
    return tc::image_bytes(lay);
}

extern "C" int ttkv_decoder_image(const ttkv_layout_t* lay, const float* decoders, int64_t dec_stride, int32_t n,
                                  void* image, int64_t image_stride, float* scales, void* stream) {
    if (!lay) return fail(TTKV_ERR_ARG, "layout is null");
    const size_t per = ttkv_decoder_image_bytes(lay);
    if (!per) return fail(TTKV_ERR_UNSUPPORTED, "the tensor-core decode does not serve r1=%d, d=%d", lay->r1, lay->d);
    if (n < 0 || (n && (!decoders || !image || !scales))) return fail(TTKV_ERR_ARG, "null decoders/image/scales");
    if (dec_stride < int64_t(lay->r1) * lay->H * kHeadDim) return fail(TTKV_ERR_ARG, "decoder stride");
    if ((reinterpret_cast<uintptr_t>(image) & 15) || (image_stride & 15) || image_stride < int64_t(per))
        return fail(TTKV_ERR_ALIGN, "image must be 16-byte aligned with a stride of at least %zu bytes", per);
    if (n == 0) return TTKV_OK;
    const int kp16 = (lay->r1 + 15) / 16 * 16;
    tc::decoder_image_kernel<<<dim3(n, lay->H), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        decoders, dec_stride, lay->r1, lay->H, kp16, (kp16 + 63) / 64, static_cast<unsigned char*>(image),
        image_stride, scales);
    return check_launch("decoder_image_kernel");
}

extern "C" int ttkv_prefill_cont_paged(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                                       const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                                       const int32_t* q_start, const int32_t* q_len, const void* q,
                                       int32_t q_dtype, int64_t q_stride, int32_t HQ, float scale,
                                       int32_t head_lo, int32_t head_hi, void* out,
                                       int32_t out_dtype, int64_t out_stride, int32_t max_q_len,
                                       int32_t max_seq_len, void* workspace,
                                       size_t workspace_bytes, int32_t* status, void* stream) {
    return read_entry(true, lay, cache, batch, rope, q_start, q_len, q, q_dtype, q_stride, HQ, scale,
                      head_lo, head_hi, out, out_dtype, out_stride, max_q_len, max_seq_len,
                      workspace, workspace_bytes, status, stream);
}

// ------------------------------------------------------------------ decode, allocation-free
// The split-K partials of ttkv_decode_paged_noalloc: a file-scope device array, one copy per GPU
// that loads the library. Host code must not take its address directly (that is a host-side
// stand-in); the device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_decode_scratch[TTKV_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;

int noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* ptrs[kMaxDevices] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(TTKV_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(TTKV_ERR_UNSUPPORTED, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || !p)
            return fail(TTKV_ERR_CUDA, "cudaGetSymbolAddress(decode scratch) on device %d: %s", dev,
                        cudaGetErrorString(e));
        ptrs[dev] = p;
    }
    *out = ptrs[dev];
    return TTKV_OK;
}
}  // namespace

extern "C" int ttkv_decode_paged_noalloc(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                                         const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                                         const void* q, int32_t q_dtype, int64_t q_stride,
                                         int32_t HQ, float scale, int32_t head_lo, int32_t head_hi,
                                         void* out, int32_t out_dtype, int64_t out_stride,
                                         int32_t max_seq_len, int32_t* status, void* stream) {
    // the same refusals as ttkv_decode_paged, before the scratch is sized (a bad argument is
    // TTKV_ERR_ARG, never TTKV_ERR_WORKSPACE)
    if (int e = check_read_args(false, lay, cache, batch, rope, nullptr, nullptr, q, q_dtype, q_stride, HQ,
                                head_lo, head_hi, out, out_dtype, out_stride, 1, max_seq_len))
        return e;
    const size_t need = decode_workspace(lay, batch->n_reqs, HQ, max_seq_len, head_lo, head_hi, cache->block_size);
    if (need > size_t(TTKV_NOALLOC_SCRATCH_BYTES))
        return fail(TTKV_ERR_WORKSPACE,
                    "this decode (%d requests, max_seq_len %d, HQ %d) needs %zu bytes of scratch but "
                    "the allocation-free entry point has %u (TTKV_NOALLOC_SCRATCH_BYTES); call "
                    "ttkv_decode_paged with a workspace instead",
                    batch->n_reqs, max_seq_len, HQ, need, TTKV_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    if (int e = noalloc_scratch(&scratch)) return e;
    return read_entry(false, lay, cache, batch, rope, nullptr, nullptr, q, q_dtype, q_stride, HQ,
                      scale, head_lo, head_hi, out, out_dtype, out_stride, 1, max_seq_len, scratch,
                      size_t(TTKV_NOALLOC_SCRATCH_BYTES), status, stream);
}

// The head-sharded decode with its outputs gathered over NVLink peer stores in the merge.
static int check_peers(const ttkv_peers_t* peers) {
    if (!peers || peers->world < 1 || peers->world > TTKV_MAX_PEERS || peers->rank < 0 ||
        peers->rank >= peers->world || !peers->epoch || !peers->ticket)
        return fail(TTKV_ERR_ARG, "peers: world %d, rank %d", peers ? peers->world : 0, peers ? peers->rank : 0);
    for (int i = 0; i < peers->world; ++i)
        if (!peers->out[i] || !peers->signal[i]) return fail(TTKV_ERR_ARG, "peers: rank %d has no out or signal", i);
    return TTKV_OK;
}

extern "C" int ttkv_decode_paged_gather(const ttkv_layout_t* lay, const ttkv_cache_t* cache,
                                        const ttkv_batch_t* batch, const ttkv_rope_t* rope,
                                        const void* q, int32_t q_dtype, int64_t q_stride, int32_t HQ,
                                        float scale, int32_t head_lo, int32_t head_hi, void* out,
                                        int32_t out_dtype, int64_t out_stride, int32_t max_seq_len,
                                        void* workspace, size_t workspace_bytes, const ttkv_peers_t* peers,
                                        int32_t* status, void* stream) {
    if (int e = check_peers(peers)) return e;
    if (peers->out[peers->rank] != out) return fail(TTKV_ERR_ARG, "peers: out[rank] is not the call's out");
    // every rank's merge must arrive: a call that would launch nothing is refused instead
    if ((batch && batch->n_reqs == 0) || max_seq_len == 0)
        return fail(TTKV_ERR_ARG, "a gathered decode of no requests or rows");
    return read_entry(false, lay, cache, batch, rope, nullptr, nullptr, q, q_dtype, q_stride, HQ, scale,
                      head_lo, head_hi, out, out_dtype, out_stride, 1, max_seq_len, workspace,
                      workspace_bytes, status, stream, peers);
}

extern "C" int ttkv_peer_wait(const ttkv_peers_t* peers, int64_t arrivals, int32_t* status, void* stream) {
    if (int e = check_peers(peers)) return e;
    if (arrivals < 1 || !status) return fail(TTKV_ERR_ARG, "arrivals %lld", (long long)arrivals);
    peer_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        peers->signal[peers->rank], peers->epoch, (unsigned long long)arrivals, status);
    return check_launch("peer_wait_kernel");
}
