// The continuation read on the tensor cores, sm_100a: S = Q . Y^T and O += P . V on tcgen05.
//
// Included by ttkv_read.cu after ttkv_decode_tc.cuh (shares ReadParams and the device helpers).
//
// A continuation chunk has many query rows per stored token, so the stored tile is rebuilt ONCE
// for a whole block of rows and every product with it runs on the tensor pipe. One CTA per
// (request, KV head, block of 128 consecutive (query, query head) rows: row i of the request's
// chunk is query i / G, head i % G, so a query's heads may sit in two blocks and a chunk of q
// queries takes ceil(q G / 128) CTAs per KV head). It walks the stored 128-token tiles the block's
// last query can see:
//
//   MMA 1   acc[128 tokens x 128 dims] = A . B_hi + A . B_lo      (as the decode: A = int8
//           coefficients as exact fp16, B = the decoder slice as fp16 hi + lo)
//   keys    k = acc * (cs 2^e) + residual, rotated by the token's position, split into hi + lo in
//           the query's dtype -> Y_hi, Y_lo [tokens x dims]; the V codes as exact fp16 integers
//           -> V [tokens x lanes]; the V ruler -> vr[token]
//   S       S[rows x tokens] = Q . Y_hi^T + Q . Y_lo^T   (Q exact in its dtype: q is the model's)
//   softmax scale, causal limit (stored row <= the query's position), online max and sum;
//           P' = p * vr split into fp16 hi + lo, written over S in tensor memory; O rescaled in
//           tensor memory when a row's max moved
//   PV      O[rows x lanes] += P'_hi . V + P'_lo . V   (A from tensor memory)
//
// and finally writes O / l for its rows. The decoder slice and Y share one buffer (the slice is
// re-staged, from L2, once S has read Y), so the plan fits with hi/lo on every inexact operand.
// No scratch and no merge: each CTA owns its rows.
//
// Threads: four epilogue warpgroups, an MMA warp and a producer warp. Epilogue thread (wg, t)
// owns TMEM lane t (a token for the keys, a row for the softmax) and a quarter of its columns, as
// the decode splits them: RoPE pairs [16wg, 16wg + 16), V lanes [32wg, 32wg + 32), stored rows
// [32wg, 32wg + 32) of the tile, output lanes [32wg, 32wg + 32). The producer warp stages each
// tile's slot fields with cp.async; lane 0 of the MMA warp issues the MMAs and the decoder copies.
// Every mbarrier wait is bounded (TTKV_STATUS_TIMEOUT).
//
// This is vllm_ttkv/impl.py:725-778 (_prefill_continuation) with krt_multi_from_slots
// (krt_triton.py:269-317), the causal softmax and v_out_multi_from_slots (v_out_triton.py:249-294).

namespace ct {

using namespace tc;

constexpr int NWGE = 4;                       // epilogue warpgroups
constexpr int NEPI = 128 * NWGE;
constexpr int NTHR = NEPI + 64;             // + the MMA warp and the producer warp
constexpr uint32_t TMEM_COLS = 512;
// tensor memory: the reconstruction, S (then P'_hi in its first 64 columns and P'_lo in the
// next 64, two 16-bit values per column), O
constexpr uint32_t ACC_COL = 0, S_COL = 128, PH_COL = 128, PL_COL = 192, O_COL = 256;
constexpr int RAW_PITCH = 144;                // raw coefficient rows: 128 B + 16 (conflict-free reads)
constexpr int CT_BT_CAP = TM + 1;             // block ids of one tile (block size 1: 128, plus one)
constexpr float LOG2E = 1.4426950408889634f;

struct CtGeom {
    int natom, kp16, cb;
    int kr, vr, kvrow;
    int bs_shift;                     // log2(block size) when it is a power of two, else -1
    int off_by, off_q, off_a, off_raw, off_v, off_kv, off_vr, off_red, off_bt, off_lut, off_misc;
    int smem;
};

struct CtMisc {
    uint64_t mb_r, mb_s, mb_pv, mb_b, mb_cf, mb_kv;       // async completions
    uint64_t mb_a, mb_y, mb_kvf, mb_p;                    // epilogue -> control
    uint32_t tmem_base;
    int bad;
};

// Instruction descriptor of a kind::f16 MMA with fp16 or bf16 operands and an fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_16(int M, int N, bool a_mn, bool b_mn, bool bf16) {
    return idesc_f16(M, N, a_mn, b_mn) | (bf16 ? ((1u << 7) | (1u << 10)) : 0u);
}

// D (+)= A . B with A read from tensor memory (lane = row, two 16-bit K values per column).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void ct_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// The epilogue warpgroups' own barrier (the control warp does not take part).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" :: "n"(NEPI) : "memory"); }

// 2^x (PTX ex2.approx: relative error about 2^-22, far inside the read's tolerance).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,"
        "%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,"
        "%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
           "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
           "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
           "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
           "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
           "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
           "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
           "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
           "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
           "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
           "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
           "r"(v[15])
        : "memory");
}

// Two 16-bit values (fp16 or bf16) of x, y, round to nearest even: the hi word and the remainder's.
__device__ __forceinline__ void split16(float x, float y, bool bf16, uint32_t& hi, uint32_t& lo) {
    if (bf16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
        const float2 hf = __bfloat1622float2(h);
        const __nv_bfloat162 l = __floats2bfloat162_rn(x - hf.x, y - hf.y);
        hi = *reinterpret_cast<const uint32_t*>(&h);
        lo = *reinterpret_cast<const uint32_t*>(&l);
    } else {
        const __half2 h = __floats2half2_rn(x, y);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
        hi = *reinterpret_cast<const uint32_t*>(&h);
        lo = *reinterpret_cast<const uint32_t*>(&l);
    }
}

// grid (row blocks, KV heads, requests), NTHR threads. q_start / q_len: the requests' query rows.
__global__ void __launch_bounds__(NTHR, 1) cont_tc_kernel(const ReadParams P, const CtGeom T) {
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    unsigned char* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    unsigned char* by = base + T.off_by;        // decoder slice hi || lo, then Y hi || lo
    unsigned char* qb = base + T.off_q;         // Q [rows x dims], K-major
    unsigned char* amat = base + T.off_a;       // coefficients as fp16, K-major
    unsigned char* raw = base + T.off_raw;      // raw coefficient blocks [token][RAW_PITCH]
    unsigned char* vb = base + T.off_v;         // V [tokens x lanes], MN-major
    unsigned char* kvb = base + T.off_kv;       // [token][K region | V region]
    float* vr_s = reinterpret_cast<float*>(base + T.off_vr);      // [tile parity][token]
    float* red = reinterpret_cast<float*>(base + T.off_red);      // [warpgroup][row]
    int32_t* bts = reinterpret_cast<int32_t*>(base + T.off_bt);   // the staged tile's block ids
    uint4* lutk = reinterpret_cast<uint4*>(base + T.off_lut);
    uint4* lutv = lutk + 16;
    CtMisc* M = reinterpret_cast<CtMisc*>(base + T.off_misc);

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const bool epi = tid < NEPI;
    const int wg = (tid >> 7) & (NWGE - 1), t = tid & 127;
    const int G = P.G;
    const int hl = int(blockIdx.y), h = P.head_lo + hl, r = int(blockIdx.z);
    const int row0 = int(blockIdx.x) * TM;                    // first (query, head) row of the block
    pdl_wait();

    // ---- the block: its queries, the stored rows its last query sees, the refusals (uniform)
    const int seq = P.seq_lens[r], ql = P.q_len[r];
    if (row0 >= ql * G) return;                              // no rows here (also for ql <= 0)
    if (ql > seq) {
        if (tid == 0 && blockIdx.x == 0 && hl == 0) report(P.status, TTKV_STATUS_QUERY);
        return;
    }
    if (seq > P.max_seq) {
        if (tid == 0 && blockIdx.x == 0 && hl == 0) report(P.status, TTKV_STATUS_SEQ_BOUND);
        return;
    }
    const int di = P.dec_index[r];
    if (di < 0 || di >= P.n_decoders) {
        if (tid == 0 && blockIdx.x == 0 && hl == 0) report(P.status, TTKV_STATUS_DECODER);
        return;
    }
    if ((seq + P.block_size - 1) / P.block_size > P.bt_cols) {
        if (tid == 0 && blockIdx.x == 0 && hl == 0) report(P.status, TTKV_STATUS_ROW_SHORT);
        return;
    }
    const int nrows = min(TM, ql * G - row0);                 // rows of this block
    const int jlast = (row0 + nrows - 1) / G;                 // the block's last query
    const int p0 = seq - ql;                                  // position of query 0
    const int limit = min(seq, p0 + jlast + 1);               // stored rows the last query sees
    const int n_tiles = (limit + TM - 1) / TM;
    const int32_t* brow = P.block_table + int64_t(r) * P.bt_stride;
    const int64_t n_blocks = P.n_slots / P.block_size;
    const bool qbf = P.q_dtype == TTKV_BF16;
    const int qrow0 = P.q_start[r];                           // the chunk's query 0 in q / out

    // ---- set-up: TMEM, barriers, shift tables
    if (w == NEPI / 32) tmem_alloc(&M->tmem_base, TMEM_COLS);
    if (tid == 0) {
        mbar_init(&M->mb_r, 1);
        mbar_init(&M->mb_s, 1);
        mbar_init(&M->mb_pv, 1);
        mbar_init(&M->mb_b, 1);
        mbar_init(&M->mb_cf, 32);
        mbar_init(&M->mb_kv, 32);
        mbar_init(&M->mb_a, NEPI);
        mbar_init(&M->mb_y, NEPI);
        mbar_init(&M->mb_kvf, NEPI);
        mbar_init(&M->mb_p, NEPI);
        M->bad = 0;
    }
    if (tid < 32) {
        const int n = tid & 15, bits = tid < 16 ? P.res_bits : P.v_bits;
        (tid < 16 ? lutk : lutv)[n] =
            make_uint4(lut_shift(n, 0, bits), lut_shift(n, 1, bits), lut_shift(n, 2, bits), lut_shift(n, 3, bits));
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t taddr = M->tmem_base;
    const uint32_t t_row = taddr + (uint32_t(32 * (w & 3)) << 16);

    const int kfield = P.coeff_bytes + 2 + h * P.k_row;
    const int vfield = P.v_offset + h * P.v_row;
    const int koff = kfield & 15, voff = vfield & 15;
    const uint32_t kbytes = uint32_t((koff + P.k_row + 15) & ~15), vbytes = uint32_t((voff + P.v_row + 15) & ~15);

    const uint32_t img_bytes = uint32_t(2 * T.natom * ATOM_BYTES);
    const unsigned char* img = P.dec_image + int64_t(di) * P.image_stride + int64_t(h) * img_bytes;
    const float s_up = P.dec_scales[int64_t(di) * P.H + h];
    bool timed_out = false;

    if (w == NEPI / 32) {
        // ============================================================== MMA warp
        uint32_t ph_a = 0, ph_y = 0, ph_p = 0, ph_b = 0, ph_s = 0, ph_pv = 0;
        uint32_t n_r = 0, n_s = 0, n_pv = 0, n_b = 0;
        bool tmo = false;
        auto cwait = [&](uint64_t* bar, uint32_t& ph) {
            if (tmo) return;
            if (!mbar_wait(bar, ph)) tmo = true; else ph ^= 1u;
        };
        const uint64_t dA = sw128_desc(smem_u32(amat), 16, 1024);
        const uint64_t dBh = sw128_desc(smem_u32(by), 16, 1024);
        const uint64_t dBl = sw128_desc(smem_u32(by + T.natom * ATOM_BYTES), 16, 1024);
        const uint64_t dQ = sw128_desc(smem_u32(qb), 16, 1024);
        const uint64_t dYh = sw128_desc(smem_u32(by), 16, 1024), dYl = sw128_desc(smem_u32(by + 2 * ATOM_BYTES), 16, 1024);
        const uint64_t dV = sw128_desc(smem_u32(vb), 1024, 2048);
        auto k16 = [](int ks) { return uint64_t(((ks >> 2) * ATOM_BYTES + (ks & 3) * 32) >> 4); };
        if (lane == 0) {
            mbar_expect_tx(&M->mb_b, img_bytes);
            bulk_g2s(by, img, img_bytes, &M->mb_b);
            ++n_b;
        }
        for (int it = 0; it < n_tiles && !tmo; ++it) {
            // MMA 1 once A(it) is converted and the decoder slice is back
            cwait(&M->mb_a, ph_a);
            if (lane == 0) cwait(&M->mb_b, ph_b);
            tmo = __any_sync(0xffffffffu, tmo);
            if (tmo) break;
            if (lane == 0) {
                tc_after();
                constexpr uint32_t ID_R = idesc_16(128, 128, false, false, false);
                for (int ks = 0; ks < T.kp16 / 16; ++ks) {
                    mma_f16(taddr + ACC_COL, dA + k16(ks), dBh + k16(ks), ID_R, ks > 0 ? 1u : 0u);
                    mma_f16(taddr + ACC_COL, dA + k16(ks), dBl + k16(ks), ID_R, 1u);
                }
                mma_commit(&M->mb_r);
                ++n_r;
            }
            __syncwarp();
            // S once Y is written, and PV (it - 1) has read P'(it - 1) from S's columns
            cwait(&M->mb_y, ph_y);
            if (it > 0) cwait(&M->mb_pv, ph_pv);
            tmo = __any_sync(0xffffffffu, tmo);
            if (tmo) break;
            if (lane == 0) {
                tc_after();
                const uint32_t ID_S = idesc_16(128, 128, false, false, qbf);
                for (int ks = 0; ks < 8; ++ks) {
                    mma_f16(taddr + S_COL, dQ + k16(ks), dYh + k16(ks), ID_S, ks > 0 ? 1u : 0u);
                    mma_f16(taddr + S_COL, dQ + k16(ks), dYl + k16(ks), ID_S, 1u);
                }
                mma_commit(&M->mb_s);
                ++n_s;
            }
            __syncwarp();
            // Y is read once S completes: the decoder slice back into the shared buffer
            cwait(&M->mb_s, ph_s);
            tmo = __any_sync(0xffffffffu, tmo);
            if (tmo) break;
            if (lane == 0 && it + 1 < n_tiles) {
                tc_after();
                mbar_expect_tx(&M->mb_b, img_bytes);
                bulk_g2s(by, img, img_bytes, &M->mb_b);
                ++n_b;
            }
            __syncwarp();
            // PV once P' is in tensor memory and O rescaled
            cwait(&M->mb_p, ph_p);
            tmo = __any_sync(0xffffffffu, tmo);
            if (tmo) break;
            if (lane == 0) {
                tc_after();
                constexpr uint32_t ID_PV = idesc_16(128, 128, false, true, false);
                for (int ks = 0; ks < 8; ++ks) {
                    const uint64_t dv = dV + uint64_t((ks * 4096) >> 4);
                    mma_f16_ts(taddr + O_COL, taddr + PH_COL + 8 * ks, dv, ID_PV, (it > 0 || ks > 0) ? 1u : 0u);
                    mma_f16_ts(taddr + O_COL, taddr + PL_COL + 8 * ks, dv, ID_PV, 1u);
                }
                mma_commit(&M->mb_pv);
                ++n_pv;
            }
            __syncwarp();
        }
        if (tmo && lane == 0) {
            // drain what was started: the last batch of each kind (every earlier one was waited for)
            if (n_r) mbar_wait(&M->mb_r, (n_r - 1) & 1u);
            if (n_s) mbar_wait(&M->mb_s, (n_s - 1) & 1u);
            if (n_pv) mbar_wait(&M->mb_pv, (n_pv - 1) & 1u);
            if (n_b) mbar_wait(&M->mb_b, (n_b - 1) & 1u);
        }
        timed_out = tmo;
    } else if (!epi) {
        // ============================================================== producer warp
        // ---- staging (producer warp). A tile's block ids are cached in shared memory first (each
        // checked against the cache; an id outside it is reported and block 0 read instead), then the
        // 16-byte chunks are copied chunk-fastest over the tile's tokens, so a warp's copies cover a
        // few consecutive slot fields rather than 32 scattered rows. Every lane arrives once per phase
        // after its own copies.
        const int bsz = P.block_size;
        auto blk_of = [&](int tok) { return T.bs_shift >= 0 ? tok >> T.bs_shift : tok / bsz; };
        auto load_bt = [&](int it) {
            const int t0 = it * TM, n = min(TM, limit - t0);
            const int b0 = blk_of(t0), nb = blk_of(t0 + n - 1) - b0 + 1;         // <= CT_BT_CAP
            for (int i = lane; i < nb; i += 32) {
                int32_t blk = brow[b0 + i];
                if (blk < 0 || blk >= n_blocks) { M->bad = 1; blk = 0; }
                bts[i] = blk;
            }
            __syncwarp();
        };
        auto slot_row = [&](int tok, int b0) -> const uint8_t* {
            const int bi = blk_of(tok);
            return P.cache + (int64_t(bts[bi - b0]) * bsz + (tok - bi * bsz)) * P.row_bytes;
        };
        const int cch = T.cb >> 4, nkvc = int(kbytes + vbytes) >> 4, kch = int(kbytes) >> 4;
        const uint32_t mul_cf = uint32_t((0x100000000ull + cch - 1) / cch);
        const uint32_t mul_kv = uint32_t((0x100000000ull + nkvc - 1) / nkvc);
        // i / d as a multiply-high (i < 2^12, so the rounding of the multiplier never reaches a
        // quotient boundary); d = 1 has no 32-bit multiplier
        auto div_small = [](uint32_t i, uint32_t mul, int d) { return d == 1 ? i : __umulhi(i, mul); };
        auto issue_cf = [&](int it) {                // the tile's block ids are in bts
            const int t0 = it * TM, n = min(TM, limit - t0), b0 = blk_of(t0);
            for (int i = lane; i < n * cch; i += 32) {
                const uint32_t u = div_small(uint32_t(i), mul_cf, cch), c = uint32_t(i) - u * uint32_t(cch);
                cp_async16(raw + u * RAW_PITCH + 16 * c, slot_row(t0 + int(u), b0) + 16 * c);
            }
            cp_async_arrive(&M->mb_cf);
        };
        auto issue_kv = [&](int it) {                // the tile's block ids are in bts
            const int t0 = it * TM, n = min(TM, limit - t0), b0 = blk_of(t0);
            for (int i = lane; i < n * nkvc; i += 32) {
                const uint32_t u = div_small(uint32_t(i), mul_kv, nkvc), c = uint32_t(i) - u * uint32_t(nkvc);
                const uint8_t* src = slot_row(t0 + int(u), b0);
                unsigned char* dst = kvb + u * T.kvrow;
                if (int(c) < kch) cp_async16(dst + 16 * c, src + (kfield - koff) + 16 * c);
                else cp_async16(dst + T.kr + 16 * (c - kch), src + (vfield - voff) + 16 * (c - kch));
            }
            cp_async_arrive(&M->mb_kv);
        };
        uint32_t ph_a = 0, ph_kvf = 0;
        bool tmo = false;
        auto pwait = [&](uint64_t* bar, uint32_t& ph) {
            if (tmo) return;
            if (!mbar_wait(bar, ph)) tmo = true; else ph ^= 1u;
        };
        load_bt(0);
        issue_cf(0);
        issue_kv(0);
        for (int it = 0; it + 1 < n_tiles && !tmo; ++it) {
            // the raw blocks of tile it are converted (A(it) arrived): the next tile's
            pwait(&M->mb_a, ph_a);
            tmo = __any_sync(0xffffffffu, tmo);
            if (tmo) break;
            load_bt(it + 1);                          // kv(it) was issued from the slice before
            issue_cf(it + 1);
            // the K/V rows of tile it are consumed (the keys and V are built): the next tile's
            pwait(&M->mb_kvf, ph_kvf);
            tmo = __any_sync(0xffffffffu, tmo);
            if (tmo) break;
            issue_kv(it + 1);
        }
        if (tmo) asm volatile("cp.async.wait_all;" ::: "memory");   // this warp's copies land first
        timed_out = tmo;
    } else {
        // ============================================================== epilogue
        uint32_t ph_cf = 0, ph_kv = 0, ph_r = 0, ph_s = 0, ph_pv = 0;
        bool tmo = false;
        auto ewait = [&](uint64_t* bar, uint32_t& ph) {
            if (tmo) return;
            if (!mbar_wait(bar, ph)) tmo = true; else ph ^= 1u;
            tmo = __any_sync(0xffffffffu, tmo);           // warp-uniform: tcgen05 ld/st are warp-wide
        };
        const int kbits = P.res_bits, vbits = P.v_bits;
        const uint32_t kflip = flip_mask(kbits), vflip = flip_mask(vbits);
        const uint32_t khalf = 1u << (kbits - 1), vhalf = 1u << (vbits - 1);
        const uint32_t kmask = (1u << kbits) - 1u, vmask2 = ((1u << vbits) - 1u) * 0x10001u;
        const uint32_t kmag = 0x4B000000u | khalf;
        const float kmag_f = 8388608.f + float(khalf);
        const uint32_t vmag2 = 0x64006400u | (vhalf * 0x10001u);
        const __half2 vbias2 = __floats2half2_rn(1024.f + float(vhalf), 1024.f + float(vhalf));
        const bool tbf16 = P.table_dtype == TTKV_BF16;
        const float sl2 = P.scale * LOG2E;                    // scores in base 2
        // this thread's row (softmax): query jq of the block, head g; its causal limit
        const int jq = (row0 + t) / G, g = row0 + t - jq * G;
        const bool row_ok = t < nrows;
        const int row_lim = row_ok ? p0 + jq + 1 : 0;            // sees stored rows < row_lim
        float m_run = -INFINITY, l_run = 0.f;

        // Q row t (query jq, head g), dims [32wg, 32wg + 32), into its operand once for all tiles
        {
            const uint4* src = reinterpret_cast<const uint4*>(
                static_cast<const uint16_t*>(P.q) + int64_t(qrow0 + (row_ok ? jq : 0)) * P.q_stride +
                int64_t(h * G + (row_ok ? g : 0)) * 128) + 4 * wg;
            uint4 qv[4];
            #pragma unroll
            for (int c = 0; c < 4; ++c) qv[c] = row_ok ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int ch = 4 * wg + c;
                *reinterpret_cast<uint4*>(qb + (ch >> 3) * ATOM_BYTES + kmajor_off(t, ch & 7)) = qv[c];
            }
        }

        // A: token t's coefficients (its raw block) as exact fp16; this warpgroup converts the
        // 16-coefficient chunks wg and wg + 4. Returns the coefficient scale x 2^e.
        auto convert_a = [&](bool valid) {
            const unsigned char* rrow = raw + t * RAW_PITCH;
            const int nc16 = T.kp16 / 16;
            const int sb = P.coeff_bytes;
            const float cs = valid ? f16_bits_to_f32(uint32_t(rrow[sb]) | (uint32_t(rrow[sb + 1]) << 8)) : 0.f;
            #pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int c16 = wg + NWGE * i;
                if (c16 >= nc16) break;
                const uint4 rw = valid ? *reinterpret_cast<const uint4*>(rrow + 16 * c16) : make_uint4(0, 0, 0, 0);
                uint32_t wds[4] = {rw.x, rw.y, rw.z, rw.w};
                const int left = P.r1 - 16 * c16;
                #pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int keep = left - 4 * k;
                    const uint32_t mask = keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : (0xffffffffu >> (8 * (4 - keep)));
                    wds[k] &= mask;
                }
                uint32_t hv[8];
                #pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t x = wds[k] ^ 0x80808080u;
                    const uint32_t lo2 = __byte_perm(x, 0x64646464u, 0x4140);
                    const uint32_t hi2 = __byte_perm(x, 0x64646464u, 0x4342);
                    const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
                    const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo2), bias);
                    const __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi2), bias);
                    hv[2 * k] = *reinterpret_cast<const uint32_t*>(&a);
                    hv[2 * k + 1] = *reinterpret_cast<const uint32_t*>(&b);
                }
                const int cidx = 2 * c16;
                *reinterpret_cast<uint4*>(amat + (cidx >> 3) * ATOM_BYTES + kmajor_off(t, cidx & 7)) =
                    make_uint4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<uint4*>(amat + ((cidx + 1) >> 3) * ATOM_BYTES + kmajor_off(t, (cidx + 1) & 7)) =
                    make_uint4(hv[4], hv[5], hv[6], hv[7]);
            }
            return cs * s_up;
        };

        ewait(&M->mb_cf, ph_cf);
        float csp = convert_a(t < limit);
        fence_async_smem();
        tc_before();
        ct_arrive(&M->mb_a);

        for (int it = 0; it < n_tiles; ++it) {
            const int t0 = it * TM;
            const int tok = t0 + t;
            const bool valid = tok < limit;
            // this token's RoPE rows for pairs [16wg, 16wg + 16): cos at 2wg + hp, sin at 8 + 2wg + hp
            uint4 cosw[2], sinw[2];
            {
                const uint4* trow = reinterpret_cast<const uint4*>(
                    reinterpret_cast<const uint16_t*>(P.table) + int64_t(min(valid ? tok : 0, int(P.table_rows - 1))) * 128);
                #pragma unroll
                for (int hp = 0; hp < 2; ++hp) {
                    cosw[hp] = __ldg(trow + 2 * wg + hp);
                    sinw[hp] = __ldg(trow + 8 + 2 * wg + hp);
                }
            }

            // ---- this token's K residual windows for its pairs, and the K ruler
            ewait(&M->mb_kv, ph_kv);
            const unsigned char* kvrow = kvb + t * T.kvrow;
            const uint32_t kv_off = uint32_t(kvrow - base);
            uint32_t kwin[4], kbyte[4];
            float krs;
            {
                const uint4* kp = reinterpret_cast<const uint4*>(kvrow);
                uint32_t bw[4];
                bitmap_words(kp[0], kp[1], koff, bw);
                if (!valid) bw[0] = bw[1] = bw[2] = bw[3] = 0u;
                trim_bitmap(bw, P.res_k);
                int pre[4];
                pre[0] = 0;
                pre[1] = __popc(bw[0]);
                pre[2] = pre[1] + __popc(bw[1]);
                pre[3] = pre[2] + __popc(bw[2]);
                #pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int grp = (q & 1 ? 8 : 0) + 2 * wg + (q >> 1);
                    kbyte[q] = bitmap_byte(bw, grp);
                    kwin[q] = window32(base, kv_off + uint32_t(koff + 16), uint32_t(byte_rank(bw, pre, grp) * kbits)) ^ kflip;
                }
                krs = valid ? f16_at(kvrow + koff + 16 + P.k_pb) : 0.f;
            }
            // ---- V of this tile needs PV (it - 1) done (it read V); so does the O rescale below
            if (it > 0) ewait(&M->mb_pv, ph_pv);
            tc_after();
            {
                // V lanes [32wg, 32wg + 32) of this token as exact small integers
                const unsigned char* vrow = kvrow + T.kr;
                const uint32_t vfo = kv_off + uint32_t(T.kr + voff);
                const uint4* vp = reinterpret_cast<const uint4*>(vrow);
                uint32_t bw[4];
                bitmap_words(vp[0], vp[1], voff, bw);
                if (!valid) bw[0] = bw[1] = bw[2] = bw[3] = 0u;
                trim_bitmap(bw, P.v_lanes);
                const uint32_t word = wg == 0 ? bw[0] : wg == 1 ? bw[1] : wg == 2 ? bw[2] : bw[3];
                const int rank0 = (wg > 0 ? __popc(bw[0]) : 0) + (wg > 1 ? __popc(bw[1]) : 0) + (wg > 2 ? __popc(bw[2]) : 0);
                #pragma unroll
                for (int gi = 0; gi < 4; ++gi) {
                    const uint32_t byte = (word >> (24 - 8 * gi)) & 0xffu;
                    const int rank = rank0 + (gi ? __popc(word >> (32 - 8 * gi)) : 0);
                    const uint32_t win = window32(base, vfo + 16u, uint32_t(rank * vbits)) ^ vflip;
                    uint32_t f[8];
                    group_fields(win, byte, vbits, lutv, f);
                    uint32_t hv[4];
                    #pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t x = (__byte_perm(f[2 * k], f[2 * k + 1], 0x5410) & vmask2) ^ vmag2;
                        const __half2 y = __hsub2(*reinterpret_cast<const __half2*>(&x), vbias2);
                        hv[k] = *reinterpret_cast<const uint32_t*>(&y);
                    }
                    const int ch = 4 * wg + gi;
                    const uint32_t off = uint32_t((t >> 3) * 2048 + (ch >> 3) * 1024 + (t & 7) * 128 +
                                                  (((ch & 7) ^ (t & 7)) << 4));
                    *reinterpret_cast<uint4*>(vb + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
                if (wg == 0) vr_s[(it & 1) * TM + t] = valid ? f16_at(vrow + voff + 16 + P.v_pb) : 0.f;
            }
            ct_arrive(&M->mb_kvf);                               // the K/V rows are read

            // ---- the keys: MMA 1 (it) done; k, RoPE, hi/lo into Y (the decoder's buffer, free now)
            ewait(&M->mb_r, ph_r);
            tc_after();
            {
                const float2 csp2 = make_float2(csp, csp), krs2 = make_float2(krs, krs);
                #pragma unroll
                for (int hp = 0; hp < 2; ++hp) {
                    const int jd = 16 * wg + 8 * hp;                  // dims jd.. and 64 + jd..
                    float al[8], ah[8];
                    tmem_ld8(t_row + ACC_COL + uint32_t(jd), al);
                    tmem_ld8(t_row + ACC_COL + uint32_t(64 + jd), ah);
                    float rl[8], rh[8];
                    {
                        uint32_t f[8];
                        group_fields(kwin[2 * hp], kbyte[2 * hp], kbits, lutk, f);
                        #pragma unroll
                        for (int k = 0; k < 8; ++k) rl[k] = __uint_as_float((f[k] & kmask) ^ kmag) - kmag_f;
                        group_fields(kwin[2 * hp + 1], kbyte[2 * hp + 1], kbits, lutk, f);
                        #pragma unroll
                        for (int k = 0; k < 8; ++k) rh[k] = __uint_as_float((f[k] & kmask) ^ kmag) - kmag_f;
                    }
                    tmem_wait_ld();
                    const uint32_t cwv[4] = {cosw[hp].x, cosw[hp].y, cosw[hp].z, cosw[hp].w};
                    const uint32_t swv[4] = {sinw[hp].x, sinw[hp].y, sinw[hp].z, sinw[hp].w};
                    uint32_t yhl[4], yll[4], yhh[4], ylh[4];              // hi/lo of y_l, y_h
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float2 cz, sz;
                        if (tbf16) {
                            cz = make_float2(__uint_as_float(cwv[i] << 16), __uint_as_float(cwv[i] & 0xffff0000u));
                            sz = make_float2(__uint_as_float(swv[i] << 16), __uint_as_float(swv[i] & 0xffff0000u));
                        } else {
                            cz = __half22float2(*reinterpret_cast<const __half2*>(&cwv[i]));
                            sz = __half22float2(*reinterpret_cast<const __half2*>(&swv[i]));
                        }
                        const float2 kl = f2fma(make_float2(rl[2 * i], rl[2 * i + 1]), krs2,
                                                f2mul(make_float2(al[2 * i], al[2 * i + 1]), csp2));
                        const float2 kh = f2fma(make_float2(rh[2 * i], rh[2 * i + 1]), krs2,
                                                f2mul(make_float2(ah[2 * i], ah[2 * i + 1]), csp2));
                        float2 yl = make_float2(fmaf(-kh.x, sz.x, kl.x * cz.x), fmaf(-kh.y, sz.y, kl.y * cz.y));
                        float2 yh = make_float2(fmaf(kl.x, sz.x, kh.x * cz.x), fmaf(kl.y, sz.y, kh.y * cz.y));
                        if (!valid) { yl = make_float2(0.f, 0.f); yh = yl; }
                        split16(yl.x, yl.y, qbf, yhl[i], yll[i]);
                        split16(yh.x, yh.y, qbf, yhh[i], ylh[i]);
                    }
                    const int ch = 2 * wg + hp;
                    *reinterpret_cast<uint4*>(by + kmajor_off(t, ch)) = make_uint4(yhl[0], yhl[1], yhl[2], yhl[3]);
                    *reinterpret_cast<uint4*>(by + ATOM_BYTES + kmajor_off(t, ch)) = make_uint4(yhh[0], yhh[1], yhh[2], yhh[3]);
                    *reinterpret_cast<uint4*>(by + 2 * ATOM_BYTES + kmajor_off(t, ch)) = make_uint4(yll[0], yll[1], yll[2], yll[3]);
                    *reinterpret_cast<uint4*>(by + 3 * ATOM_BYTES + kmajor_off(t, ch)) = make_uint4(ylh[0], ylh[1], ylh[2], ylh[3]);
                }
            }
            fence_async_smem();
            tc_before();
            ct_arrive(&M->mb_y);                                  // Y and V written; the accumulator read

            // ---- the next tile's coefficients into A (MMA 1 (it) has read it)
            if (it + 1 < n_tiles) {
                ewait(&M->mb_cf, ph_cf);
                csp = convert_a(t0 + TM + t < limit);
                fence_async_smem();
                tc_before();
                ct_arrive(&M->mb_a);
            }

            // ---- softmax of row t over stored rows [32wg, 32wg + 32) of the tile; P' hi / lo
            ewait(&M->mb_s, ph_s);
            tc_after();
            // every V ruler of this tile is written, and every reduction slot of the tile before
            // read (the rulers are double-buffered by tile: a thread writes tile it + 2's only
            // after this barrier of tile it + 1, which follows every read of tile it's)
            epi_sync();
            {
                const float* vrt = vr_s + (it & 1) * TM + 32 * wg;
                float sv[32];
                tmem_ld32(t_row + S_COL + uint32_t(32 * wg), sv);
                tmem_wait_ld();
                float mt = -INFINITY;
                const int c0 = t0 + 32 * wg;                      // the stored row of sv[0]
                if (__all_sync(0xffffffffu, c0 + 32 <= row_lim)) {      // no row of the warp is cut here
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) { sv[i] *= sl2; mt = fmaxf(mt, sv[i]); }
                } else {
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        sv[i] = c0 + i < row_lim ? sv[i] * sl2 : -INFINITY;
                        mt = fmaxf(mt, sv[i]);
                    }
                }
                red[wg * TM + t] = mt;
                epi_sync();                                        // every S column is read too
                const float tmax = fmaxf(fmaxf(red[t], red[TM + t]), fmaxf(red[2 * TM + t], red[3 * TM + t]));
                const float m_new = fmaxf(m_run, tmax);
                // nothing seen yet: O and l are zero, nothing to rescale
                const float corr = (m_run == -INFINITY) ? 1.f : ex2(m_run - m_new);
                float lsum = 0.f;
                uint32_t phi[16], plo[16];
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 va = reinterpret_cast<const float4*>(vrt)[2 * c];
                    const float4 vb4 = reinterpret_cast<const float4*>(vrt)[2 * c + 1];
                    const float vrc[8] = {va.x, va.y, va.z, va.w, vb4.x, vb4.y, vb4.z, vb4.w};
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float pp[2];
                        #pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            const int tt = 8 * c + 2 * i + k;
                            const float pg = sv[tt] == -INFINITY ? 0.f : ex2(sv[tt] - m_new);
                            lsum += pg;
                            pp[k] = pg * vrc[2 * i + k];
                        }
                        const __half2 hh = __floats2half2_rn(pp[0], pp[1]);
                        const float2 hf = __half22float2(hh);
                        const __half2 ll = __floats2half2_rn(pp[0] - hf.x, pp[1] - hf.y);
                        phi[4 * c + i] = *reinterpret_cast<const uint32_t*>(&hh);
                        plo[4 * c + i] = *reinterpret_cast<const uint32_t*>(&ll);
                    }
                }
                // P' over S: stored rows 32wg.. are columns 16wg.. of each half
                tmem_st16u(t_row + PH_COL + uint32_t(16 * wg), phi);
                tmem_st16u(t_row + PL_COL + uint32_t(16 * wg), plo);
                l_run = l_run * corr + lsum;                       // this warpgroup's share of the sum
                // O lanes [32wg, 32wg + 32) (after PV (it - 1), waited above) rescaled where a max moved
                if (it > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
                    float o32[32];
                    tmem_ld32(t_row + O_COL + uint32_t(32 * wg), o32);
                    tmem_wait_ld();
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) o32[i] *= corr;
                    tmem_st32(t_row + O_COL + uint32_t(32 * wg), o32);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                m_run = m_new;
            }
            tc_before();
            ct_arrive(&M->mb_p);
            // no early exit after a timeout: every epilogue warp runs every tile's named barriers
            // (its waits return at once), so the barrier counts stay equal across the warpgroups
        }
        // ---- the output rows: O / l after the last PV (l summed over the warpgroups' shares)
        if (!tmo) {
            ewait(&M->mb_pv, ph_pv);
            tc_after();
        }
        epi_sync();                                                // the last tile's max slots are read
        red[wg * TM + t] = l_run;
        epi_sync();
        const float l = (red[t] + red[TM + t]) + (red[2 * TM + t] + red[3 * TM + t]);
        if (!tmo) {
            // every lane loads (tcgen05.ld is warp-wide); rows past the block's queries store nothing
            const float inv = l > 0.f ? 1.f / l : 0.f;
            const int64_t ob = int64_t(qrow0 + (row_ok ? jq : 0)) * P.out_stride + int64_t(h * G + g) * 128 + 32 * wg;
            float o32[32];
            tmem_ld32(t_row + O_COL + uint32_t(32 * wg), o32);
            tmem_wait_ld();
            if (row_ok) {
                #pragma unroll
                for (int i = 0; i < 32; ++i) store_elt(P.out, P.out_dtype, ob + i, o32[i] * inv);
            }
        }
        timed_out = tmo;
    }
    if (__syncthreads_or(timed_out) && tid == 0) report(P.status, TTKV_STATUS_TIMEOUT);
    if (tid == 0 && M->bad) report(P.status, TTKV_STATUS_BLOCK_RANGE);
    tc_before();
    __syncthreads();
    tc_after();
    if (w == NEPI / 32) tmem_dealloc(M->tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ host plan
// The shared-memory plan of cont_tc_kernel, or smem == 0 where it does not fit (layouts with
// more than two 64-rank atoms, or a coefficient block of more than 128 bytes, use the decode path).
inline CtGeom ct_geom(const ttkv_layout_t* lay, int G, int block_size) {
    CtGeom T{};
    T.kp16 = round_up(lay->r1, 16);
    T.natom = (T.kp16 + 63) / 64;
    T.cb = round_up(lay->coeff_bytes + 2, 16);
    T.bs_shift = -1;
    for (int s = 0; s < 31; ++s)
        if (block_size == (1 << s)) T.bs_shift = s;
    int kr = 0, vr = 0;
    for (int hh = 0; hh < lay->H; ++hh) {
        const int kf = lay->coeff_bytes + 2 + hh * lay->k_row_bytes;
        const int vf = lay->v_offset + hh * lay->v_row_bytes;
        kr = std::max(kr, round_up((kf & 15) + lay->k_row_bytes, 16));
        vr = std::max(vr, round_up((vf & 15) + lay->v_row_bytes, 16));
    }
    T.kr = std::max(kr, 32);
    T.vr = std::max(vr, 32);
    T.kvrow = T.kr + T.vr;
    if (((T.kvrow >> 4) & 1) == 0) T.kvrow += 16;
    if (T.natom > 2 || T.cb > 128) { T.smem = 0; return T; }
    int off = 0;
    T.off_by = off; off += std::max(2 * T.natom * ATOM_BYTES, 4 * ATOM_BYTES);
    T.off_q = off; off += 2 * ATOM_BYTES;
    T.off_a = off; off += T.natom * ATOM_BYTES;
    T.off_v = off; off += APV_BYTES;
    T.off_raw = off; off += TM * RAW_PITCH;
    T.off_kv = off; off += TM * T.kvrow + KV_PAD;
    off = round_up(off, 16);
    T.off_vr = off; off += 2 * TM * 4;
    T.off_red = off; off += NWGE * TM * 4;
    T.off_bt = off; off += round_up(CT_BT_CAP * 4, 16);
    T.off_lut = off; off += LUT_BYTES;
    T.off_misc = off; off += round_up(int(sizeof(CtMisc)), 16);
    T.smem = round_up(off, 16) + 1024;
    if (T.smem > 227 * 1024) T.smem = 0;
    return T;
}

}  // namespace ct
