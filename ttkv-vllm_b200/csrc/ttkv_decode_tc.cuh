// The decode read on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Included by ttkv_read.cu inside its anonymous namespace (shares ReadParams and the merge).
//
// One CTA = (request, KV head, token split), 128 threads; thread t owns token t of the current
// 128-token tile, which is also TMEM lane t. Per tile:
//
//   stage    cp.async (16 B) of each token's coefficient block, this head's K residual row and V
//            row into shared memory, double-buffered across tiles
//   A        coefficients int8 -> fp16 (exact) in the canonical K-major SW128 layout
//   MMA 1    acc[128 tokens x 128 lanes] = A . B_hi + A . B_lo  (fp32 in TMEM), where B is the
//            head's slice of the request's decoder, pre-scaled by a power of two and split into
//            fp16 hi + lo so the product is accurate to ~2^-22 (a single fp16 operand moved
//            attention outputs by 4.4e-4 on the parity store; bf16 by 2.7e-3)
//   epilogue per token: k = acc * (cs * 2^e) + residual lanes; RoPE by the token's own position;
//            scores of the G query heads; online softmax over the tile
//   MMA 2    O^T[128 lanes x 16] += V^T . P', V^T = the tile's V codes (exact small integers in
//            fp16, MN-major so each token writes its row contiguously), P' = p * V ruler split
//            into hi (columns 0..G-1) and lo (columns G..2G-1)
//
// Every wait on an mbarrier is bounded (a clock limit); a timeout sets TTKV_STATUS_TIMEOUT, drains
// what is in flight, frees TMEM and returns. No wait depends on another CTA.

namespace tc {

constexpr int TM = 128;                 // tokens per tile = UMMA M = TMEM lanes
constexpr int NTHR = 128;
constexpr uint32_t TMEM_COLS = 256;     // power of two >= 128 (recon) + 16 (PV)
constexpr uint32_t PV_COL = 128;
constexpr int ATOM_BYTES = 128 * 128;   // one SW128 K-major atom column: 128 rows x 128 B
constexpr int APV_BYTES = 32768;        // V^T: 128 tokens x 128 lanes fp16
constexpr int BPV_BYTES = 4096;         // P': 16 rows x 128 tokens fp16
constexpr long long WAIT_CYCLES = 4000000000LL;   // ~2 s at 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory matrix descriptor for tcgen05 (start, LBO, SBO in 16-byte units; version 1;
// layout type 2 = 128-byte swizzle). Field positions follow the sm_100 UMMA descriptor.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor, kind::f16 with fp16 A/B and an fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait for an mbarrier phase: false after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > WAIT_CYCLES) return false;
    return true;
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst)), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Byte offset of (row, 16-byte chunk) in a K-major SW128 atom column of 128-byte rows.
__device__ __forceinline__ uint32_t kmajor_off(int row, int chunk) {
    return uint32_t((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// fp16 bits of (code - offset), exact for |code - offset| <= 2048.
__device__ __forceinline__ uint32_t small_int_f16(int v) {
    return f16_bits(float(v));
}

struct TcGeom {            // host-computed shared-memory plan
    int natom, nstage;     // K atoms of 64 ranks; staging buffers
    int kp16;              // r1 rounded up to 16 (the MMA K extent)
    int cb, kr, vr, srow;  // staged bytes per token: coefficient block, K region, V region, total
    int off_bhi, off_blo, off_a, off_apv, off_bpv, off_stage, off_q, off_misc;
    int smem;              // dynamic shared memory requested (includes 1 KB alignment slack)
};

struct TcMisc {
    float red_max[4][kMaxG];
    float red_sum[4][kMaxG];
    float m[kMaxG];
    float l[kMaxG];
    float maxabs[4];
    uint64_t mbar;
    uint32_t tmem_base;
    int32_t flag;
};

template <int G>
__global__ void __launch_bounds__(NTHR, 1) decode_tc_kernel(const ReadParams P, const TcGeom T) {
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    unsigned char* bhi = base + T.off_bhi;
    unsigned char* blo = base + T.off_blo;
    unsigned char* amat = base + T.off_a;
    unsigned char* apv = base + T.off_apv;
    unsigned char* bpv = base + T.off_bpv;
    unsigned char* stage0 = base + T.off_stage;
    float* qs = reinterpret_cast<float*>(base + T.off_q);
    TcMisc* M = reinterpret_cast<TcMisc*>(base + T.off_misc);

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, hl = blockIdx.y, r = blockIdx.z;
    const int h = P.head_lo + hl;
    const int seq = P.seq_lens[r];
    const int QG = G;                                           // decode: one query row per head

    // ---- validation (uniform across the CTA)
    const int di = P.dec_index[r];
    bool bad = false;
    if (di < 0 || di >= P.n_decoders) { report(P.status, TTKV_STATUS_DECODER); bad = true; }
    const int blocks_needed = (seq + P.block_size - 1) / P.block_size;
    if (!bad && blocks_needed > P.bt_cols) { report(P.status, TTKV_STATUS_ROW_SHORT); bad = true; }
    const int t_begin = split * P.chunk;
    const int t_end = min(seq, t_begin + P.chunk);
    const int32_t* brow = P.block_table + int64_t(r) * P.bt_stride;
    if (!bad && t_begin < t_end) {
        const int64_t n_blocks = P.n_slots / P.block_size;
        int local_bad = 0;
        for (int b = t_begin / P.block_size + tid; b <= (t_end - 1) / P.block_size; b += NTHR) {
            const int32_t blk = brow[b];
            if (blk < 0 || blk >= n_blocks) local_bad = 1;
        }
        if (__syncthreads_or(local_bad)) {
            if (tid == 0) report(P.status, TTKV_STATUS_BLOCK_RANGE);
            bad = true;
        }
    }
    const int64_t row_base = (int64_t(r) * P.n_heads + hl) * QG;
    if (bad || t_begin >= t_end) {
        if (tid < QG) {
            P.part_ml[((row_base + tid) * P.n_splits + split) * 2 + 0] = -INFINITY;
            P.part_ml[((row_base + tid) * P.n_splits + split) * 2 + 1] = 0.f;
        }
        for (int g = 0; g < QG; ++g) P.part_o[((row_base + g) * P.n_splits + split) * 128 + tid] = 0.f;
        return;
    }

    // ---- set-up: TMEM, barrier, operands that live for the whole CTA
    if (w == 0) tmem_alloc(&M->tmem_base, TMEM_COLS);
    if (tid == 0) { mbar_init(&M->mbar, 1); M->flag = 0; }
    if (tid < kMaxG) { M->m[tid] = -INFINITY; M->l[tid] = 0.f; }
    for (int i = tid; i < BPV_BYTES / 16; i += NTHR) reinterpret_cast<uint4*>(bpv)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < G * 128; i += NTHR) {
        const int g = i >> 7, j = i & 127;
        qs[i] = load_elt(P.q, P.q_dtype, int64_t(r) * P.q_stride + int64_t(h * G + g) * 128 + j);
    }
    // decoder slice: power-of-two scale so max|D| * 2^-e lies in [2^13, 2^14), then fp16 hi + lo
    const float* dec = P.decoders + int64_t(di) * P.dec_stride + h * 128 + tid;
    const int64_t dstride = int64_t(P.H) * 128;
    float mx = 0.f;
    for (int rr = 0; rr < P.r1; ++rr) mx = fmaxf(mx, fabsf(dec[rr * dstride]));
    mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
    if (lane == 0) M->maxabs[w] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(M->maxabs[0], M->maxabs[1]), fmaxf(M->maxabs[2], M->maxabs[3]));
    int e = 0;
    if (mx > 0.f) e = int((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 13;
    e = max(-100, min(100, e));
    const float s_down = __uint_as_float(uint32_t(127 - e) << 23);   // 2^-e
    const float s_up = __uint_as_float(uint32_t(127 + e) << 23);     // 2^e
    for (int cidx = 0; cidx < T.kp16 / 8; ++cidx) {
        uint32_t hw[4], lw[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t hh[2], ll[2];
            #pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int rr = cidx * 8 + 2 * i + k;
                const float v = rr < P.r1 ? dec[rr * dstride] * s_down : 0.f;
                hh[k] = f16_bits(v);
                ll[k] = f16_bits(v - f16_bits_to_f32(hh[k]));
            }
            hw[i] = hh[0] | (hh[1] << 16);
            lw[i] = ll[0] | (ll[1] << 16);
        }
        const uint32_t off = uint32_t((cidx >> 3) * ATOM_BYTES) + kmajor_off(tid, cidx & 7);
        *reinterpret_cast<uint4*>(bhi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(blo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }

    // ---- staging of one tile: 16-byte chunks of each token's three regions
    const int kfield = P.coeff_bytes + 2 + h * P.k_row;
    const int vfield = P.v_offset + h * P.v_row;
    const int koff = kfield & 15, voff = vfield & 15;
    // chunks this head needs: exactly the 16-byte blocks covering each field, never past the blob
    const int cch = T.cb >> 4;
    const int kch = (koff + P.k_row + 15) >> 4, vch = (voff + P.v_row + 15) >> 4;
    const int nch = cch + kch + vch;
    auto issue_stage = [&](int t0, unsigned char* st) {
        const int ntok = min(TM, t_end - t0);
        for (int i = tid; i < ntok * nch; i += NTHR) {
            const int t = i / nch, c = i - t * nch;
            const int tok = t0 + t;
            const int64_t slot = int64_t(brow[tok / P.block_size]) * P.block_size + tok % P.block_size;
            const uint8_t* src = P.cache + slot * P.row_bytes;
            int gofs, sofs;
            if (c < cch) {
                gofs = c * 16;
                sofs = c * 16;
            } else if (c < cch + kch) {
                gofs = (kfield - koff) + (c - cch) * 16;
                sofs = T.cb + (c - cch) * 16;
            } else {
                gofs = (vfield - voff) + (c - cch - kch) * 16;
                sofs = T.cb + T.kr + (c - cch - kch) * 16;
            }
            cp_async16(st + t * T.srow + sofs, src + gofs);
        }
        cp_async_commit();
    };

    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t taddr = M->tmem_base;
    const uint32_t t_row = taddr + (uint32_t(32 * w) << 16);     // this warp's TMEM lanes

    constexpr uint32_t IDESC_R = idesc_f16(128, 128, false, false);
    constexpr uint32_t IDESC_PV = idesc_f16(128, 16, true, false);
    const float kbias = float(1 << (P.res_bits - 1));
    const int voffset = 1 << (P.v_bits - 1);

    float o[G];
    #pragma unroll
    for (int g = 0; g < G; ++g) o[g] = 0.f;
    uint32_t phase = 0;
    bool timed_out = false;

    issue_stage(t_begin, stage0);
    int it = 0;
    for (int t0 = t_begin; t0 < t_end; t0 += TM, ++it) {
        unsigned char* st = stage0 + size_t(T.nstage == 2 ? (it & 1) : 0) * (TM * T.srow);
        cp_async_wait_all();
        __syncthreads();
        if (T.nstage == 2 && t0 + TM < t_end)
            issue_stage(t0 + TM, stage0 + size_t((it + 1) & 1) * (TM * T.srow));

        const int tok = t0 + tid;
        const bool valid = tok < t_end;
        const unsigned char* srow = st + tid * T.srow;

        // ---- A: this token's coefficients as fp16, zero past r1 (and for an invalid token).
        // int8 -> fp16 exactly: flip the sign bit (b + 128 as a byte), place the byte under the
        // fp16 exponent of 1024 (0x64__ = 1024 + byte), subtract 1152.
        for (int c16 = 0; c16 < T.kp16 / 16; ++c16) {
            uint4 raw = valid ? *reinterpret_cast<const uint4*>(srow + 16 * c16) : make_uint4(0, 0, 0, 0);
            const int left = P.r1 - 16 * c16;                       // coefficient bytes in this chunk
            uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int keep = left - 4 * i;                      // bytes of this word that are coefficients
                const uint32_t mask = keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : (0xffffffffu >> (8 * (4 - keep)));
                wds[i] &= mask;
            }
            uint32_t hv[8];
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t x = wds[i] ^ 0x80808080u;
                const uint32_t lo2 = __byte_perm(x, 0x64646464u, 0x4140);   // bytes 0,1 -> two halves
                const uint32_t hi2 = __byte_perm(x, 0x64646464u, 0x4342);   // bytes 2,3
                const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
                const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo2), bias);
                const __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi2), bias);
                hv[2 * i] = *reinterpret_cast<const uint32_t*>(&a);
                hv[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&b);
            }
            const int cidx = 2 * c16;
            *reinterpret_cast<uint4*>(amat + (cidx >> 3) * ATOM_BYTES + kmajor_off(tid, cidx & 7)) =
                make_uint4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<uint4*>(amat + ((cidx + 1) >> 3) * ATOM_BYTES + kmajor_off(tid, (cidx + 1) & 7)) =
                make_uint4(hv[4], hv[5], hv[6], hv[7]);
        }
        // ---- V^T (MN-major): this token's V lanes as exact small integers, zero if invalid
        const unsigned char* vrow = srow + T.cb + T.kr + voff;
        uint32_t vw[4], vpre[4];
        {
            uint32_t acc = 0;
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                vw[i] = valid ? bitmap_word(vrow, i) : 0u;
                vpre[i] = acc;
                acc += __popc(vw[i]);
            }
        }
        const float vrs = valid ? f16_at(vrow + 16 + P.v_pb) : 0.f;
        #pragma unroll 1
        for (int ch = 0; ch < 16; ++ch) {
            const int wi = ch >> 2;
            const uint32_t word = wi == 0 ? vw[0] : wi == 1 ? vw[1] : wi == 2 ? vw[2] : vw[3];
            const uint32_t pre = wi == 0 ? vpre[0] : wi == 1 ? vpre[1] : wi == 2 ? vpre[2] : vpre[3];
            uint32_t wv[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t hh[2];
                #pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int l = ((ch & 3) << 3) + 2 * i + k;          // lane within the word
                    int v = 0;
                    if ((word >> (31 - l)) & 1u) {
                        const int rank = int(pre) + __popc(word & ~(0xffffffffu >> l));
                        if (rank < P.v_lanes) v = code_at(vrow + 16, rank, P.v_bits) - voffset;
                    }
                    hh[k] = small_int_f16(v);
                }
                wv[i] = hh[0] | (hh[1] << 16);
            }
            // token tid = K index, lanes 8ch..8ch+7 = one 16-byte chunk along MN
            const uint32_t off = uint32_t((tid >> 3) * 2048 + (ch >> 3) * 1024 + (tid & 7) * 128 +
                                          (((ch & 7) ^ (tid & 7)) << 4));
            *reinterpret_cast<uint4*>(apv + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        fence_async_smem();
        tc_before();
        __syncthreads();
        tc_after();

        // ---- MMA 1: reconstruction
        if (tid == 0) {
            const uint32_t a0 = smem_u32(amat), h0 = smem_u32(bhi), l0 = smem_u32(blo);
            for (int ks = 0; ks < T.kp16 / 16; ++ks) {
                const uint32_t kofs = uint32_t((ks >> 2) * ATOM_BYTES + (ks & 3) * 32);
                const uint64_t ad = sw128_desc(a0 + kofs, 16, 1024);
                mma_f16(taddr, ad, sw128_desc(h0 + kofs, 16, 1024), IDESC_R, ks > 0 ? 1u : 0u);
                mma_f16(taddr, ad, sw128_desc(l0 + kofs, 16, 1024), IDESC_R, 1u);
            }
            mma_commit(&M->mbar);
        }

        // ---- while the MMA runs: this token's K residual row, ruler, position
        const unsigned char* krow = srow + T.cb + koff;
        uint32_t kw[4], kpre[4];
        {
            uint32_t acc = 0;
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                kw[i] = valid ? bitmap_word(krow, i) : 0u;
                kpre[i] = acc;
                acc += __popc(kw[i]);
            }
        }
        const float krs = valid ? f16_at(krow + 16 + P.k_pb) : 0.f;
        const float csp = (valid ? f16_at(srow + P.coeff_bytes) : 0.f) * s_up;
        const int pos = valid ? tok : t_begin;
        const uint16_t* trow = reinterpret_cast<const uint16_t*>(P.table) +
                               int64_t(min(pos, int(P.table_rows - 1))) * 128;
        const bool tbf16 = P.table_dtype == TTKV_BF16;

        if (!mbar_wait(&M->mbar, phase)) timed_out = true;
        phase ^= 1u;
        if (__syncthreads_or(timed_out)) break;
        tc_after();

        // ---- epilogue: rebuild, patch, rotate, score
        float s[G];
        #pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        #pragma unroll 1
        for (int c = 0; c < 2; ++c) {
            float alo[32], ahi[32];
            uint4 cs4[4], sn4[4];                                   // 32 cos + 32 sin, 16-bit
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                cs4[i] = __ldg(reinterpret_cast<const uint4*>(trow + 32 * c) + i);
                sn4[i] = __ldg(reinterpret_cast<const uint4*>(trow + 64 + 32 * c) + i);
            }
            tmem_ld32(t_row + uint32_t(32 * c), alo);
            tmem_ld32(t_row + uint32_t(64 + 32 * c), ahi);
            tmem_wait_ld();
            // lanes 32c.. live in bitmap word c, lanes 64+32c.. in word c+2
            const uint32_t wl = c == 0 ? kw[0] : kw[1], wh = c == 0 ? kw[2] : kw[3];
            const uint32_t pl = c == 0 ? kpre[0] : kpre[1], ph = c == 0 ? kpre[2] : kpre[3];
            #pragma unroll
            for (int l = 0; l < 32; ++l) {
                const int jl = 32 * c + l, jh = jl + 64;
                float rl = 0.f, rh = 0.f;
                if ((wl >> (31 - l)) & 1u) {
                    const int rank = int(pl) + __popc(wl & ~(0xffffffffu >> l));
                    if (rank < P.res_k) rl = (float(code_at(krow + 16, rank, P.res_bits)) - kbias) * krs;
                }
                if ((wh >> (31 - l)) & 1u) {
                    const int rank = int(ph) + __popc(wh & ~(0xffffffffu >> l));
                    if (rank < P.res_k) rh = (float(code_at(krow + 16, rank, P.res_bits)) - kbias) * krs;
                }
                const float klo = fmaf(alo[l], csp, rl);
                const float khi = fmaf(ahi[l], csp, rh);
                const uint32_t cw = reinterpret_cast<const uint32_t*>(&cs4[l >> 3])[(l >> 1) & 3];
                const uint32_t sw = reinterpret_cast<const uint32_t*>(&sn4[l >> 3])[(l >> 1) & 3];
                const uint32_t cb = (l & 1) ? (cw >> 16) : (cw & 0xffffu);
                const uint32_t sb = (l & 1) ? (sw >> 16) : (sw & 0xffffu);
                const float cz = tbf16 ? __uint_as_float(cb << 16) : f16_bits_to_f32(cb);
                const float sz = tbf16 ? __uint_as_float(sb << 16) : f16_bits_to_f32(sb);
                const float ylo = klo * cz - khi * sz;
                const float yhi = khi * cz + klo * sz;
                #pragma unroll
                for (int g = 0; g < G; ++g)
                    s[g] = fmaf(qs[g * 128 + jl], ylo, fmaf(qs[g * 128 + jh], yhi, s[g]));
            }
        }

        // ---- online softmax over the tile
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            s[g] = valid ? s[g] * P.scale : -INFINITY;
            float mxg = s[g];
            #pragma unroll
            for (int off = 16; off; off >>= 1) mxg = fmaxf(mxg, __shfl_xor_sync(0xffffffffu, mxg, off));
            if (lane == 0) M->red_max[w][g] = mxg;
        }
        __syncthreads();
        float corr[G], m_new[G];
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            const float tmax = fmaxf(fmaxf(M->red_max[0][g], M->red_max[1][g]),
                                     fmaxf(M->red_max[2][g], M->red_max[3][g]));
            const float m_old = M->m[g];
            m_new[g] = fmaxf(m_old, tmax);
            const float pg = (m_new[g] == -INFINITY || s[g] == -INFINITY) ? 0.f : expf(s[g] - m_new[g]);
            corr[g] = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new[g]);
            float sum = pg;
            #pragma unroll
            for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (lane == 0) M->red_sum[w][g] = sum;
            // P' = p * V ruler as fp16 hi (column g) + lo (column G + g); this token is K index tid
            const float pv = pg * vrs;
            const uint32_t hb = f16_bits(pv);
            const uint32_t lb = f16_bits(pv - f16_bits_to_f32(hb));
            const int kt = tid & 63, atom = tid >> 6;
            #pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int n = k == 0 ? g : G + g;
                const uint32_t off = uint32_t(atom * 2048 + (n >> 3) * 1024 + (n & 7) * 128 +
                                              (((kt >> 3) ^ (n & 7)) << 4) + (kt & 7) * 2);
                *reinterpret_cast<uint16_t*>(bpv + off) = uint16_t(k == 0 ? hb : lb);
            }
        }
        fence_async_smem();
        tc_before();
        __syncthreads();
        tc_after();

        // ---- MMA 2: O^T[lane][col] += V^T . P'  (8 K-steps of 16 tokens)
        if (tid == 0) {
            const uint32_t a0 = smem_u32(apv), b0 = smem_u32(bpv);
            for (int ks = 0; ks < TM / 16; ++ks) {
                const uint64_t ad = sw128_desc(a0 + uint32_t(ks * 4096), 1024, 2048);
                const uint64_t bd = sw128_desc(b0 + uint32_t((ks >> 2) * 2048 + (ks & 3) * 32), 16, 1024);
                mma_f16(taddr + PV_COL, ad, bd, IDESC_PV, ks > 0 ? 1u : 0u);
            }
            mma_commit(&M->mbar);
        }
        // running max / sum: thread g owns query head g's state (every thread read M->m above)
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            if (tid == g) {
                float tsum = M->red_sum[0][g] + M->red_sum[1][g] + M->red_sum[2][g] + M->red_sum[3][g];
                M->l[g] = M->l[g] * corr[g] + tsum;
                M->m[g] = m_new[g];
            }
        }
        if (!mbar_wait(&M->mbar, phase)) timed_out = true;
        phase ^= 1u;
        if (__syncthreads_or(timed_out)) break;
        tc_after();
        {
            float d[16];
            tmem_ld16(t_row + PV_COL, d);
            tmem_wait_ld();
            #pragma unroll
            for (int g = 0; g < G; ++g) o[g] = fmaf(o[g], corr[g], d[g] + d[G + g]);
        }
        tc_before();
        if (T.nstage == 1 && t0 + TM < t_end) {
            __syncthreads();                               // the single stage buffer is free
            issue_stage(t0 + TM, stage0);
        }
    }

    // ---- drain and release: a timed-out MMA gets one more bounded wait before TMEM is freed
    if (timed_out) {
        if (tid == 0) report(P.status, TTKV_STATUS_TIMEOUT);
        mbar_wait(&M->mbar, phase ^ 1u);
    }
    cp_async_wait_all();
    tc_before();
    __syncthreads();
    tc_after();
    if (w == 0) tmem_dealloc(taddr, TMEM_COLS);
    #pragma unroll
    for (int g = 0; g < G; ++g)
        P.part_o[((row_base + g) * P.n_splits + split) * 128 + tid] = timed_out ? 0.f : o[g];
    if (tid < G) {
        P.part_ml[((row_base + tid) * P.n_splits + split) * 2 + 0] = timed_out ? -INFINITY : M->m[tid];
        P.part_ml[((row_base + tid) * P.n_splits + split) * 2 + 1] = timed_out ? 0.f : M->l[tid];
    }
}

// ------------------------------------------------------------------ host plan
inline int round_up(int x, int a) { return (x + a - 1) / a * a; }

// The shared-memory plan of decode_tc_kernel for a layout, or smem == 0 if it does not fit.
inline TcGeom tc_geom(const ttkv_layout_t* lay, int G) {
    TcGeom T{};
    T.kp16 = round_up(lay->r1, 16);
    T.natom = (T.kp16 + 63) / 64;
    T.cb = round_up(lay->coeff_bytes + 2, 16);
    int kr = 0, vr = 0;
    for (int h = 0; h < lay->H; ++h) {
        const int kf = lay->coeff_bytes + 2 + h * lay->k_row_bytes;
        const int vf = lay->v_offset + h * lay->v_row_bytes;
        kr = std::max(kr, round_up((kf & 15) + lay->k_row_bytes, 16));
        vr = std::max(vr, round_up((vf & 15) + lay->v_row_bytes, 16));
    }
    T.kr = kr;
    T.vr = vr;
    T.srow = T.cb + kr + vr;
    const int atoms = T.natom * ATOM_BYTES;
    const int q_bytes = round_up(G * 128 * 4, 1024);
    const int misc = round_up(int(sizeof(TcMisc)), 128);
    for (int ns = 2; ns >= 1; --ns) {
        int off = 0;
        T.off_bhi = off; off += atoms;
        T.off_blo = off; off += atoms;
        T.off_a = off; off += atoms;
        T.off_apv = off; off += APV_BYTES;
        T.off_bpv = off; off += BPV_BYTES;
        T.off_q = off; off += q_bytes;
        T.off_misc = off; off += misc;
        T.off_stage = off; off += ns * TM * T.srow;
        T.nstage = ns;
        T.smem = off + 1024;
        if (T.smem <= 227 * 1024) return T;
    }
    T.smem = 0;
    return T;
}

}  // namespace tc
