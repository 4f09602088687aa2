// The token-wide decode read on the tensor cores (tcgen05 + TMEM), sm_100a.
//
// Included by ttkv_read.cu after ttkv_decode_tc.cuh, inside its namespaces: it shares ReadParams,
// the schedule (units, virtual shares, partial slots), the merge and the device helpers of the
// quarter-lane kernel there, which keeps serving the layouts this one does not fit.
//
// Why a second kernel. In decode_tc_kernel four warpgroups split each token's 128 head lanes, so
// every per-token cost that does not scale with lanes (the bitmaps, the rulers, the softmax, the
// partial-score exchange, the barriers) is paid four times per token, and the SIMT issue slots,
// not HBM, bound the read. Here two threads own a (token, KV head): each decodes 64 residual lanes
// and 64 V lanes and scores its half of the rotation pairs for all G query heads; they exchange one
// partial score per query head, and both run the token's softmax.
//
// Roles. Threads 0..255 (eight warps; warps w and w + 4 share TMEM lanes 32 (w & 3) ..) are the
// epilogue: threads t and 128 + t are token t of the current 128-token tile, each with half of the
// head's lanes (a quarter of the old kernel's per-token overhead, half its code per thread), their
// partial scores summed through shared memory. Warp 8 is the control warp: its 32 lanes stage the tile's slot fields
// with 16-byte cp.async (chunk-fastest over the tokens), and its lane 0 issues the MMAs. The two
// sides meet only on mbarriers:
//
//   epilogue (tile j)                                      control, on each hand-off
//   ----------------------------------------------------  ------------------------------------------
//   wait K/V rows (j): bitmaps, code windows, rulers
//   wait MMA 1 (j); coefficients (j+1) -> A -> A ready     MMA 1 (j+1); coefficients (j+2) staged
//   k = acc * (cs 2^e) + residual, RoPE, scores            (MMA 1 (j+1) runs under this epilogue)
//   wait PV (j-1) (long done): fold it into o
//   V codes -> V^T (fp16 integers)          -> K/V free    K/V rows of tile j+2 (or j+1) into it
//   partial scores exchanged, tile max, p, P' -> PV ready  PV (j)
//
//   MMA 1   acc[128 tokens x 128 lanes] = A . B_hi + A . B_lo in TMEM (two column sets, so MMA 1 of
//           the next tile runs under this tile's epilogue), A = int8 coefficients as exact fp16, B =
//           the head's decoder slice scaled by 2^-e and split into fp16 hi + lo (accurate to about
//           2^-22; a single fp16 operand moved attention outputs by up to 9e-4 at 1082 tokens)
//   MMA 2   O^T[128 lanes x 16] = V^T . P', P' = p * V ruler split into hi and lo columns
//
// Every mbarrier wait is bounded; a timeout is made uniform over the epilogue at the tile barrier
// (a reduction), the control warp sees it on its own bounded waits, the CTA records
// TTKV_STATUS_TIMEOUT, drains what it started and frees TMEM. No wait depends on another CTA.

namespace tw {

using namespace tc;

constexpr int NEPI = 256;                 // epilogue threads: two per token of the tile
constexpr int NTHR = NEPI + 32;           // + the control warp
constexpr uint32_t TMEM_COLS = 512;       // 2 x 128 reconstruction columns + 16 PV columns
constexpr uint32_t PV_COL = 256;
constexpr int EPI_BAR = 1;                // named barrier of the epilogue warps

struct TwGeom {            // host-computed shared-memory plan
    int natom, kp16;
    int cb, cf_pitch, cf_swz;
    int kr, vr, kvrow, nkv;
    int off_bhi, off_blo, off_a, off_apv, off_bpv, off_q, off_lut, off_misc, off_bt, off_cf, off_kv, off_xs;
    int smem;
};

struct TwMisc {
    float red_max[2][NEPI / 32][kMaxG];      // tile maxima per warp, double-buffered by tile parity
    float red_sum[NEPI / 32][kMaxG];
    float maxabs[NEPI / 32];
    int scan[NTHR / 32];
    int lim[kMaxG];
    int sched_r;
    long long sched_before;
    long long sched_T, sched_nv, sched_hi;
    uint64_t mb_r, mb_pv, mb_cf, mb_kv[2], mb_dec;   // completions of the async work
    uint64_t mb_a, mb_cff, mb_kvf[2], mb_pvr;        // epilogue -> control hand-offs
    uint32_t tmem_base;
};

// OR of `pred` over the epilogue's 128 threads; also a barrier among them.
__device__ __forceinline__ bool epi_any(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r) : "r"(uint32_t(pred)), "n"(EPI_BAR), "n"(NEPI) : "memory");
    return r != 0;
}

__device__ __forceinline__ void epi_sync() {
    asm volatile("bar.sync %0, %1;" :: "n"(EPI_BAR), "n"(NEPI) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// Exclusive prefix sum of v over the CTA's N threads in thread order, and the total. Every thread
// of the CTA calls it; `wsum` holds N / 32 ints of shared memory.
template <int N>
__device__ __forceinline__ int cta_scan_n(int v, int* wsum, int& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    int pre = 0;
    total = 0;
    #pragma unroll
    for (int i = 0; i < N / 32; ++i) {
        const int sw = wsum[i];
        if (i < w) pre += sw;
        total += sw;
    }
    __syncthreads();
    return pre + x - v;
}

template <int G>
__global__ void __launch_bounds__(NTHR, 1) decode_tw_kernel(const ReadParams P, const TwGeom T) {
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    unsigned char* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    unsigned char* bhi = base + T.off_bhi;
    unsigned char* blo = base + T.off_blo;
    unsigned char* amat = base + T.off_a;
    unsigned char* apv = base + T.off_apv;
    unsigned char* bpv = base + T.off_bpv;
    float* qs = reinterpret_cast<float*>(base + T.off_q);        // [g][pair i2][q_2i2, q_2i2+1, q_64+2i2, q_65+2i2]
    uint4* lutk = reinterpret_cast<uint4*>(base + T.off_lut);
    uint4* lutv = lutk + 16;
    TwMisc* M = reinterpret_cast<TwMisc*>(base + T.off_misc);
    unsigned char* cfb = base + T.off_cf;                         // [token][cf_pitch]
    unsigned char* kvb = base + T.off_kv;                         // [buffer][token][K region | V region]
    int32_t* bts = reinterpret_cast<int32_t*>(base + T.off_bt);
    float* xs = reinterpret_cast<float*>(base + T.off_xs);        // [half][g][token] partial scores

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const bool epi = tid < NEPI;
    const int t = tid & 127;                                      // epilogue: token / TMEM lane
    const int half = (tid >> 7) & 1;                              // epilogue: which half of the lanes
    const int nh = P.n_heads;
    pdl_wait();

    // ---- the schedule (as decode_tc_kernel): CTA c takes units [c T / n, (c+1) T / n)
    int64_t T_units, lo, hi;
    if (P.n_reqs <= NTHR) {
        const int v = tid < P.n_reqs ? req_tiles(P.seq_lens[tid]) : 0;
        int tot;
        const int ex = cta_scan_n<NTHR>(v, M->scan, tot);
        T_units = int64_t(tot) * nh;
        lo = int64_t(blockIdx.x) * T_units / gridDim.x;
        hi = int64_t(blockIdx.x + 1) * T_units / gridDim.x;
        if (tid < P.n_reqs && int64_t(ex) * nh <= lo && lo < int64_t(ex + v) * nh) {
            M->sched_r = tid;
            M->sched_before = ex;
        }
    } else {
        int64_t tiles_all = 0;
        for (int b0 = 0; b0 < P.n_reqs; b0 += NTHR) {
            const int i = b0 + tid;
            int tot;
            cta_scan_n<NTHR>(i < P.n_reqs ? req_tiles(P.seq_lens[i]) : 0, M->scan, tot);
            tiles_all += tot;
        }
        T_units = tiles_all * nh;
        lo = int64_t(blockIdx.x) * T_units / gridDim.x;
        hi = int64_t(blockIdx.x + 1) * T_units / gridDim.x;
        int64_t acc = 0;
        for (int b0 = 0; b0 < P.n_reqs && acc * nh <= lo; b0 += NTHR) {
            const int i = b0 + tid;
            const int v = i < P.n_reqs ? req_tiles(P.seq_lens[i]) : 0;
            int tot;
            const int ex = cta_scan_n<NTHR>(v, M->scan, tot);
            if (i < P.n_reqs && (acc + ex) * nh <= lo && lo < (acc + ex + v) * nh) {
                M->sched_r = i;
                M->sched_before = acc + ex;
            }
            acc += tot;
        }
    }
    const int64_t nv = int64_t(gridDim.x) * virtual_shares(T_units, gridDim.x, P.block_size);
    if (tid == 0) { M->sched_T = T_units; M->sched_nv = nv; M->sched_hi = hi; }
    __syncthreads();
    pdl_trigger();
    if (nv + int64_t(P.n_reqs) * nh > P.n_part_slots) {
        if (blockIdx.x == 0 && tid == 0) report(P.status, TTKV_STATUS_SEQ_BOUND);
        return;
    }
    if (lo >= hi) return;
    int r = M->sched_r;
    int64_t before = M->sched_before;
    int64_t unit = lo;
    auto share_of = [&](int64_t u, int64_t& v, int64_t& v_end) {
        const int64_t Tn = M->sched_T, n = M->sched_nv;
        v = ((u + 1) * n - 1) / Tn;
        v_end = (v + 1) * Tn / n;
    };
    auto empty_partial = [&](int64_t slot) {
        if (tid < G) {
            P.part_ml[(slot * G + tid) * 2 + 0] = -INFINITY;
            P.part_ml[(slot * G + tid) * 2 + 1] = 0.f;
        }
        if (epi)
            for (int g = 0; g < G; ++g) P.part_o[(slot * G + g) * 128 + t] = 0.f;
    };

    // ---- CTA set-up: TMEM, barriers, shift tables, the zero columns of P'
    if (w == NEPI / 32) tmem_alloc(&M->tmem_base, TMEM_COLS);
    if (tid == 0) {
        mbar_init(&M->mb_r, 1);
        mbar_init(&M->mb_pv, 1);
        mbar_init(&M->mb_cf, 32);
        mbar_init(&M->mb_kv[0], 32);
        mbar_init(&M->mb_kv[1], 32);
        mbar_init(&M->mb_dec, 1);
        mbar_init(&M->mb_a, NEPI);
        mbar_init(&M->mb_cff, NEPI);
        mbar_init(&M->mb_kvf[0], NEPI);
        mbar_init(&M->mb_kvf[1], NEPI);
        mbar_init(&M->mb_pvr, NEPI);
    }
    if (tid < 32) {
        const int n = tid & 15, bits = tid < 16 ? P.res_bits : P.v_bits;
        (tid < 16 ? lutk : lutv)[n] =
            make_uint4(lut_shift(n, 0, bits), lut_shift(n, 1, bits), lut_shift(n, 2, bits), lut_shift(n, 3, bits));
    }
    for (int i = tid; i < BPV_BYTES / 16; i += NTHR) reinterpret_cast<uint4*>(bpv)[i] = make_uint4(0, 0, 0, 0);
    fence_async_smem();
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t taddr = M->tmem_base;
    const uint32_t t_row = taddr + (uint32_t(32 * (w & 3)) << 16);      // epilogue warp's TMEM lanes

    // phase parities: each side tracks the barriers it waits on
    uint32_t ph_r = 0, ph_pv = 0, ph_cf = 0, ph_kv0 = 0, ph_kv1 = 0;          // epilogue
    uint32_t ph_a = 0, ph_cff = 0, ph_kvf0 = 0, ph_kvf1 = 0, ph_pvr = 0, ph_dec = 0;   // control
    // the control warp's lane 0 counts the MMA batches it committed: a timeout drains the last ones
    uint32_t n_r = 0, n_pv = 0;
    bool pend_dec = false;
    bool timed_out = false;

    const int kbits = P.res_bits, vbits = P.v_bits;
    const uint32_t kflip = flip_mask(kbits), vflip = flip_mask(vbits);
    const uint32_t khalf = 1u << (kbits - 1), vhalf = 1u << (vbits - 1);
    const uint32_t kmask = (1u << kbits) - 1u, vmask2 = ((1u << vbits) - 1u) * 0x10001u;
    const uint32_t kmag = 0x4B000000u | khalf;                     // float 2^23 + code
    const float kmag_f = 8388608.f + float(khalf);
    const uint32_t vmag2 = 0x64006400u | (vhalf * 0x10001u);       // fp16 pair 1024 + code
    const __half2 vbias2 = __floats2half2_rn(1024.f + float(vhalf), 1024.f + float(vhalf));
    const bool tbf16 = P.table_dtype == TTKV_BF16;
    const float4* qs4 = reinterpret_cast<const float4*>(qs);

    const uint64_t dA = sw128_desc(smem_u32(amat), 16, 1024), dH = sw128_desc(smem_u32(bhi), 16, 1024),
                   dL = sw128_desc(smem_u32(blo), 16, 1024);
    const uint64_t dV = sw128_desc(smem_u32(apv), 1024, 2048), dP = sw128_desc(smem_u32(bpv), 16, 1024);

    while (unit < M->sched_hi && !timed_out) {
        // ---- the next segment (uniform over the CTA)
        if (r >= P.n_reqs) break;
        const int seq = P.seq_lens[r];
        const int nt = req_tiles(seq);
        const int64_t rs = before * nh, re = rs + int64_t(nt) * nh;
        if (unit >= re) { before += nt; ++r; continue; }
        int64_t vs, vs_end;
        share_of(unit, vs, vs_end);
        const int hl = int((unit - rs) / nt);
        const int64_t ps = rs + int64_t(hl) * nt;
        const int64_t seg_hi = min(vs_end, ps + nt);
        const int t_begin = int(unit - ps) * TM;
        const int t_end = min(seq, int(seg_hi - ps) * TM);
        const int64_t slot = vs + int64_t(r) * nh + hl;
        unit = seg_hi;
        const int h = P.head_lo + hl;
        const int rq = P.v_req ? P.v_req[r] : r;
        const int di = P.dec_index[rq];
        bool bad = false;
        if (seq > P.max_seq) { if (tid == 0) report(P.status, TTKV_STATUS_SEQ_BOUND); bad = true; }
        if (!bad && (di < 0 || di >= P.n_decoders)) { if (tid == 0) report(P.status, TTKV_STATUS_DECODER); bad = true; }
        const int blocks_needed = (seq + P.block_size - 1) / P.block_size;
        if (!bad && blocks_needed > P.bt_cols) { if (tid == 0) report(P.status, TTKV_STATUS_ROW_SHORT); bad = true; }
        const int32_t* brow = P.block_table + int64_t(rq) * P.bt_stride;
        if (!bad && (t_end - 1) / P.block_size - t_begin / P.block_size + 1 > BT_CAP) {
            if (tid == 0) report(P.status, TTKV_STATUS_ROW_SHORT);
            bad = true;
        }
        const int n_tiles = (t_end - t_begin + TM - 1) / TM;

        // staging geometry of this head's fields (as decode_tc_kernel)
        const int kfield = P.coeff_bytes + 2 + h * P.k_row;
        const int vfield = P.v_offset + h * P.v_row;
        const int koff = kfield & 15, voff = vfield & 15;
        const int cch = T.cb >> 4;
        const int kch = (koff + P.k_row + 15) >> 4, vch = (voff + P.v_row + 15) >> 4;
        const uint32_t bsz = uint32_t(P.block_size);
        const uint64_t mul_bs = (0x100000000ull + bsz - 1) / bsz;
        const int blk0 = t_begin / P.block_size;
        // the slot row of token `tok` of this segment (its block from the cached block-table slice)
        auto row_at = [&](int tok) -> const uint8_t* {
            const uint32_t blk = uint32_t((uint64_t(uint32_t(tok)) * mul_bs) >> 32);
            return P.cache + (int64_t(bts[int(blk) - blk0]) * P.block_size + int64_t(uint32_t(tok) - blk * bsz)) *
                             P.row_bytes;
        };
        auto ntok = [&](int tile) { return tile < n_tiles ? min(TM, t_end - (t_begin + tile * TM)) : 0; };
        // control lanes only. Lane l stages tokens l, l + 32, l + 64, l + 96 of the tile: the row
        // address once per token, then the field's 16-byte chunks; one arrival per lane per phase
        auto issue_cf = [&](int tile) {
            const int t0k = t_begin + tile * TM, n = ntok(tile);
            for (int u = lane; u < n; u += 32) {
                const uint8_t* src = row_at(t0k + u);
                unsigned char* dst = cfb + u * T.cf_pitch;
                const int swz = u & T.cf_swz;
                for (int c = 0; c < cch; ++c) cp_async16(dst + 16 * (c ^ swz), src + 16 * c);
            }
            cp_async_arrive(&M->mb_cf);
        };
        auto issue_kv = [&](int tile) {
            const int b = T.nkv == 2 ? (tile & 1) : 0, t0k = t_begin + tile * TM, n = ntok(tile);
            unsigned char* dstb = kvb + size_t(b) * TM * T.kvrow;
            for (int u = lane; u < n; u += 32) {
                const uint8_t* src = row_at(t0k + u);
                unsigned char* dst = dstb + u * T.kvrow;
                for (int c = 0; c < kch; ++c) cp_async16(dst + 16 * c, src + (kfield - koff) + 16 * c);
                for (int c = 0; c < vch; ++c) cp_async16(dst + T.kr + 16 * c, src + (vfield - voff) + 16 * c);
            }
            cp_async_arrive(&M->mb_kv[b]);
        };

        // ---- set-up pass: the block-table slice (checked), the queries, the causal row limits
        int local_bad = 0;
        if (!bad) {
            const int nblk = (t_end - 1) / P.block_size - blk0 + 1;
            const int64_t n_blocks = P.n_slots / P.block_size;
            for (int i = tid; i < nblk; i += NTHR) {
                const int32_t blk = brow[blk0 + i];
                if (blk < 0 || blk >= n_blocks) local_bad = 1;
                bts[i] = blk;
            }
            for (int i = tid; i < G * 128; i += NTHR) {
                const int g = i >> 7, j = i & 127;
                const int qi = (g * 32 + ((j & 63) >> 1)) * 4 + (j >= 64 ? 2 : 0) + (j & 1);
                float qv = 0.f;
                if (!P.v_req) {
                    qv = load_elt(P.q, P.q_dtype, int64_t(r) * P.q_stride + int64_t(h * G + g) * 128 + j);
                } else if (g < P.v_nq[r]) {
                    const int f = P.v_f0[r] + g, jq = f / P.g_real, gh = f - jq * P.g_real;
                    qv = load_elt(P.q, P.q_dtype, int64_t(P.v_qrow[r] + jq) * P.q_stride +
                                                  int64_t(h * P.g_real + gh) * 128 + j);
                }
                qs[qi] = qv;
            }
        }
        if (tid < kMaxG) {
            int lim = 0x7fffffff;
            if (P.v_req) lim = tid < P.v_nq[r] ? P.v_pos[r] + (P.v_f0[r] + tid) / P.g_real + 1 : 0;
            M->lim[tid] = lim;
        }
        if (__syncthreads_or(local_bad)) {
            if (tid == 0) report(P.status, TTKV_STATUS_BLOCK_RANGE);
            bad = true;
        }
        if (bad) {
            empty_partial(slot);
            __syncthreads();
            continue;
        }

        if (!epi) {
            // ================================================================ control warp
            issue_cf(0);
            issue_kv(0);
            if (T.nkv == 2 && n_tiles > 1) issue_kv(1);
            if (P.dec_image && lane == 0) {
                const uint32_t bytes = uint32_t(2 * T.natom * ATOM_BYTES);
                mbar_expect_tx(&M->mb_dec, bytes);
                bulk_g2s(bhi, P.dec_image + int64_t(di) * P.image_stride + int64_t(h) * bytes, bytes, &M->mb_dec);
                pend_dec = true;
            }
            bool tmo = false;
            auto cwait = [&](uint64_t* bar, uint32_t& ph) {
                if (tmo) return;
                if (!mbar_wait(bar, ph)) tmo = true; else ph ^= 1u;
            };
            // MMA 1 of tile j, and the coefficients of tile j + 1 into the buffer it frees, as soon as
            // the epilogue has converted A(j) (which also means it is done with the reconstruction
            // columns MMA 1 (j) writes, last read in tile j - 2)
            auto recon = [&](int j) {
                cwait(&M->mb_a, ph_a);
                cwait(&M->mb_cff, ph_cff);
                if (j == 0 && pend_dec) {
                    cwait(&M->mb_dec, ph_dec);
                    if (!tmo) pend_dec = false;
                }
                tmo = __any_sync(0xffffffffu, tmo);
                if (tmo) return;
                if (lane == 0) {
                    tc_after();
                    constexpr uint32_t IDESC_R = idesc_f16(128, 128, false, false);
                    const uint32_t d_tmem = taddr + uint32_t(j & 1) * 128u;
                    for (int ks = 0; ks < T.kp16 / 16; ++ks) {
                        const uint64_t k16 = uint64_t(((ks >> 2) * ATOM_BYTES + (ks & 3) * 32) >> 4);
                        mma_f16(d_tmem, dA + k16, dH + k16, IDESC_R, ks > 0 ? 1u : 0u);
                        mma_f16(d_tmem, dA + k16, dL + k16, IDESC_R, 1u);
                    }
                    mma_commit(&M->mb_r);
                    ++n_r;
                }
                __syncwarp();
                if (j + 1 < n_tiles) issue_cf(j + 1);
            };
            // the control loop follows the epilogue's hand-offs of tile j in the order they come:
            // A(j + 1) converted, K/V rows consumed, V^T and P' written
            recon(0);
            for (int j = 0; j < n_tiles && !tmo; ++j) {
                if (j + 1 < n_tiles) {
                    recon(j + 1);
                    if (tmo) break;
                }
                if (T.nkv == 2) {
                    if (j & 1) cwait(&M->mb_kvf[1], ph_kvf1); else cwait(&M->mb_kvf[0], ph_kvf0);
                    tmo = __any_sync(0xffffffffu, tmo);
                    if (tmo) break;
                    if (j + 2 < n_tiles) issue_kv(j + 2);
                } else {
                    cwait(&M->mb_kvf[0], ph_kvf0);
                    tmo = __any_sync(0xffffffffu, tmo);
                    if (tmo) break;
                    if (j + 1 < n_tiles) issue_kv(j + 1);
                }
                cwait(&M->mb_pvr, ph_pvr);
                tmo = __any_sync(0xffffffffu, tmo);
                if (tmo) break;
                if (lane == 0) {
                    tc_after();
                    constexpr uint32_t IDESC_PV = idesc_f16(128, 16, true, false);
                    #pragma unroll
                    for (int ks = 0; ks < TM / 16; ++ks)
                        mma_f16(taddr + PV_COL, dV + uint64_t((ks * 4096) >> 4),
                                dP + uint64_t(((ks >> 2) * 2048 + (ks & 3) * 32) >> 4), IDESC_PV, ks > 0 ? 1u : 0u);
                    mma_commit(&M->mb_pv);
                    ++n_pv;
                }
                __syncwarp();
            }
            timed_out = tmo;
        } else {
            // ================================================================ epilogue
            // thread (half, t): token t of the tile, RoPE pairs [32 half, 32 half + 32) -- the K
            // lanes [32 half, +32) and [64 + 32 half, +32), bitmap bytes 4 half .. 4 half + 3 and
            // 8 + 4 half .. -- and the V lanes [64 half, 64 half + 64), bitmap bytes 8 half .. + 7
            bool tmo = false;
            auto ewait = [&](uint64_t* bar, uint32_t& ph) {
                if (tmo) return;
                if (!mbar_wait(bar, ph)) tmo = true; else ph ^= 1u;
            };
            float s_up;
            if (P.dec_image) {
                s_up = P.dec_scales[int64_t(di) * P.H + h];
            } else {
                // the decoder slice converted here: column t, power-of-two scale, fp16 hi + lo; the
                // 8-row chunks split between the halves
                const float* dec = P.decoders + int64_t(di) * P.dec_stride + h * 128 + t;
                const int64_t dstride = int64_t(P.H) * 128;
                float mx = 0.f;
                for (int rr = half; rr < P.r1; rr += 2) mx = fmaxf(mx, fabsf(dec[rr * dstride]));
                mx = warp_max(mx);
                if (lane == 0) M->maxabs[w] = mx;
                epi_sync();
                mx = 0.f;
                #pragma unroll
                for (int i = 0; i < NEPI / 32; ++i) mx = fmaxf(mx, M->maxabs[i]);
                int e = 0;
                if (mx > 0.f) e = int((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 13;
                e = max(-100, min(100, e));
                const float s_down = __uint_as_float(uint32_t(127 - e) << 23);
                s_up = __uint_as_float(uint32_t(127 + e) << 23);
                for (int cidx = half; cidx < T.kp16 / 8; cidx += 2) {
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
                    const uint32_t off = uint32_t((cidx >> 3) * ATOM_BYTES) + kmajor_off(t, cidx & 7);
                    *reinterpret_cast<uint4*>(bhi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(blo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
            }

            // A: token t's coefficients as exact fp16 (int8 -> 1024 + byte under the fp16 exponent,
            // minus 1152), zero past r1 and for a token past the segment, 16-coefficient chunks
            // split between the halves; returns the token's ruler
            auto convert_a = [&](bool valid) {
                const unsigned char* srow = cfb + t * T.cf_pitch;
                const int swz = t & T.cf_swz;
                for (int c16 = half; c16 < T.kp16 / 16; c16 += 2) {
                    uint4 raw = valid ? *reinterpret_cast<const uint4*>(srow + 16 * (c16 ^ swz)) : make_uint4(0, 0, 0, 0);
                    const int left = P.r1 - 16 * c16;
                    uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
                    if (left < 16) {
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int keep = left - 4 * i;
                            const uint32_t mask = keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : (0xffffffffu >> (8 * (4 - keep)));
                            wds[i] &= mask;
                        }
                    }
                    uint32_t hv[8];
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t x = wds[i] ^ 0x80808080u;
                        const uint32_t lo2 = __byte_perm(x, 0x64646464u, 0x4140);
                        const uint32_t hi2 = __byte_perm(x, 0x64646464u, 0x4342);
                        const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
                        const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo2), bias);
                        const __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi2), bias);
                        hv[2 * i] = *reinterpret_cast<const uint32_t*>(&a);
                        hv[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&b);
                    }
                    const int cidx = 2 * c16;
                    *reinterpret_cast<uint4*>(amat + (cidx >> 3) * ATOM_BYTES + kmajor_off(t, cidx & 7)) =
                        make_uint4(hv[0], hv[1], hv[2], hv[3]);
                    *reinterpret_cast<uint4*>(amat + ((cidx + 1) >> 3) * ATOM_BYTES + kmajor_off(t, (cidx + 1) & 7)) =
                        make_uint4(hv[4], hv[5], hv[6], hv[7]);
                }
                auto byte_at = [&](int b) { return uint32_t(srow[16 * ((b >> 4) ^ swz) + (b & 15)]); };
                const int sb = P.coeff_bytes;
                return valid ? f16_bits_to_f32(byte_at(sb) | (byte_at(sb + 1) << 8)) : 0.f;
            };

            // ---- A(0): the segment's first coefficients
            ewait(&M->mb_cf, ph_cf);
            float csp_next = convert_a(t_begin + t < t_end) * s_up;
            fence_async_smem();
            tc_before();
            mbar_arrive(&M->mb_a);
            mbar_arrive(&M->mb_cff);

            float o[G], lsum[G], m_run[G], corr_prev[G];
            #pragma unroll
            for (int g = 0; g < G; ++g) { o[g] = 0.f; lsum[g] = 0.f; m_run[g] = -INFINITY; corr_prev[g] = 0.f; }
            int lim[G];
            #pragma unroll
            for (int g = 0; g < G; ++g) lim[g] = M->lim[g];
            const float scale = P.scale;

            for (int it = 0; it < n_tiles; ++it) {
                const int t0 = t_begin + it * TM;
                const int tok = t0 + t;
                const bool valid = tok < t_end;
                const bool has_next = it + 1 < n_tiles;
                const int kb = T.nkv == 2 ? (it & 1) : 0;
                const float csp = csp_next;

                // ---- this token's RoPE row for this half's pairs (cos | sin), read early from L2
                // (16 bytes of cos and of sin per 8 pairs; the first chunk's now, each next one a chunk
                // ahead of its use, so only two chunks are held in registers at a time)
                const uint4* trow = reinterpret_cast<const uint4*>(
                    reinterpret_cast<const uint16_t*>(P.table) +
                    int64_t(min(valid ? tok : t_begin, int(P.table_rows - 1))) * 128) + 4 * half;
                uint4 cos_next = __ldg(trow), sin_next = __ldg(trow + 8);

                // ---- K residual: bitmap, and the code windows of this half's 8 bitmap bytes
                if (kb) ewait(&M->mb_kv[1], ph_kv1); else ewait(&M->mb_kv[0], ph_kv0);
                const unsigned char* kvrow = kvb + (size_t(kb) * TM + t) * T.kvrow;
                const uint32_t kv_off = uint32_t(kvrow - base);
                uint32_t kbw[4], kwin[8];
                float krs;
                {
                    const uint4* kp = reinterpret_cast<const uint4*>(kvrow);
                    bitmap_words(kp[0], kp[1], koff, kbw);
                    if (!valid) kbw[0] = kbw[1] = kbw[2] = kbw[3] = 0u;
                    trim_bitmap(kbw, P.res_k);
                    int pre[4];
                    pre[0] = 0;
                    pre[1] = __popc(kbw[0]);
                    pre[2] = pre[1] + __popc(kbw[1]);
                    pre[3] = pre[2] + __popc(kbw[2]);
                    #pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        const int gb = (q4 < 4 ? 0 : 8) + 4 * half + (q4 & 3);
                        kwin[q4] = window32(base, kv_off + uint32_t(koff + 16), uint32_t(byte_rank(kbw, pre, gb) * kbits)) ^ kflip;
                    }
                    krs = valid ? f16_at(kvrow + koff + 16 + P.k_pb) : 0.f;
                }


                // ---- MMA 1 of this tile done: A takes the next tile's coefficients
                ewait(&M->mb_r, ph_r);
                tc_after();
                if (has_next) {
                    ewait(&M->mb_cf, ph_cf);
                    csp_next = convert_a(t0 + TM + t < t_end) * s_up;
                    fence_async_smem();
                    tc_before();
                    mbar_arrive(&M->mb_a);
                    mbar_arrive(&M->mb_cff);
                }

                // ---- rebuild, patch, rotate, score this half's pairs: 8 pairs (j, j + 64) at a time
                float2 s2[G], s2h[G];
                #pragma unroll
                for (int g = 0; g < G; ++g) { s2[g] = make_float2(0.f, 0.f); s2h[g] = s2[g]; }
                {
                    const uint32_t rcol = uint32_t(it & 1) * 128u;
                    const float2 csp2 = make_float2(csp, csp), krs2 = make_float2(krs, krs);
                    #pragma unroll
                    for (int hp = 0; hp < 4; ++hp) {
                        const int j0 = 32 * half + 8 * hp;
                        float al[8], ah[8];
                        tmem_ld8(t_row + rcol + uint32_t(j0), al);
                        tmem_ld8(t_row + rcol + uint32_t(64 + j0), ah);
                        float rl[8], rh[8];
                        {
                            uint32_t f[8];
                            group_fields(kwin[hp], bitmap_byte(kbw, 4 * half + hp), kbits, lutk, f);
                            #pragma unroll
                            for (int k = 0; k < 8; ++k) rl[k] = __uint_as_float((f[k] & kmask) ^ kmag);
                            group_fields(kwin[4 + hp], bitmap_byte(kbw, 8 + 4 * half + hp), kbits, lutk, f);
                            #pragma unroll
                            for (int k = 0; k < 8; ++k) rh[k] = __uint_as_float((f[k] & kmask) ^ kmag);
                        }
                        tmem_wait_ld();
                        const uint4 cw = cos_next, sw = sin_next;
                        if (hp < 3) { cos_next = __ldg(trow + hp + 1); sin_next = __ldg(trow + 9 + hp); }
                        const uint32_t cwv[4] = {cw.x, cw.y, cw.z, cw.w};
                        const uint32_t swv[4] = {sw.x, sw.y, sw.z, sw.w};
                        const float2 mag2 = make_float2(-kmag_f, -kmag_f);
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
                            // residual codes as exact floats (magic 2^23 + code, minus the magic)
                            const float2 rl2 = f2add(make_float2(rl[2 * i], rl[2 * i + 1]), mag2);
                            const float2 rh2 = f2add(make_float2(rh[2 * i], rh[2 * i + 1]), mag2);
                            const float2 kl = f2fma(rl2, krs2, f2mul(make_float2(al[2 * i], al[2 * i + 1]), csp2));
                            const float2 kh = f2fma(rh2, krs2, f2mul(make_float2(ah[2 * i], ah[2 * i + 1]), csp2));
                            const float2 yl = f2sub(f2mul(kl, cz), f2mul(kh, sz));
                            const float2 yh = f2fma(kl, sz, f2mul(kh, cz));
                            #pragma unroll
                            for (int g = 0; g < G; ++g) {
                                const float4 qq = qs4[g * 32 + (j0 >> 1) + i];
                                s2[g] = f2fma(make_float2(qq.x, qq.y), yl, s2[g]);
                                s2h[g] = f2fma(make_float2(qq.z, qq.w), yh, s2h[g]);
                            }
                        }
                    }
                }
                tc_before();        // this tile's reconstruction columns are read (next use: tile it + 2)

                // ---- PV of the previous tile: this thread is head lane t of every query head
                if (it > 0) {
                    ewait(&M->mb_pv, ph_pv);
                    tc_after();
                    float pvv[16];
                    tmem_ld16(t_row + PV_COL, pvv);
                    tmem_wait_ld();
                    #pragma unroll
                    for (int g = 0; g < G; ++g) o[g] = fmaf(o[g], corr_prev[g], pvv[g] + pvv[G + g]);
                }

                // ---- V^T (MN-major): this half's 64 lanes of the token as exact small integers
                float vrs;
                {
                    const unsigned char* vrow = kvrow + T.kr;
                    const uint32_t vfo = kv_off + uint32_t(T.kr + voff);
                    const uint4* vp = reinterpret_cast<const uint4*>(vrow);
                    uint32_t bw[4];
                    bitmap_words(vp[0], vp[1], voff, bw);
                    if (!valid) bw[0] = bw[1] = bw[2] = bw[3] = 0u;
                    trim_bitmap(bw, P.v_lanes);
                    int rank0 = half ? __popc(bw[0]) + __popc(bw[1]) : 0;
                    #pragma unroll
                    for (int wq = 0; wq < 2; ++wq) {
                        const uint32_t word = half ? bw[2 + wq] : bw[wq];
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
                            const int ch = 8 * half + 4 * wq + gi;
                            const uint32_t off = uint32_t((t >> 3) * 2048 + (ch >> 3) * 1024 + (t & 7) * 128 +
                                                          (((ch & 7) ^ (t & 7)) << 4));
                            *reinterpret_cast<uint4*>(apv + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                        }
                        rank0 += __popc(word);
                    }
                    vrs = valid ? f16_at(vrow + voff + 16 + P.v_pb) : 0.f;
                }
                mbar_arrive(&M->mb_kvf[kb]);                       // the K/V rows are in registers / V^T

                // ---- the two halves' partial scores, then the online softmax over the tile. The
                // first barrier is a reduction that also makes a timeout anywhere in the epilogue
                // everyone's; the maxima are double-buffered by tile parity
                #pragma unroll
                for (int g = 0; g < G; ++g) xs[(half * kMaxG + g) * 128 + t] = (s2[g].x + s2h[g].x) + (s2[g].y + s2h[g].y);
                if (epi_any(tmo)) { tmo = true; break; }
                float sc[G];
                #pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float v = xs[g * 128 + t] + xs[(kMaxG + g) * 128 + t];       // same order in both halves
                    sc[g] = (valid && tok < lim[g]) ? v * scale : -INFINITY;
                    const float mxg = warp_max(sc[g]);
                    if (lane == 0) M->red_max[it & 1][w][g] = mxg;
                }
                epi_sync();
                #pragma unroll
                for (int g = 0; g < G; ++g) {
                    float tmax = M->red_max[it & 1][0][g];
                    #pragma unroll
                    for (int i = 1; i < NEPI / 32; ++i) tmax = fmaxf(tmax, M->red_max[it & 1][i][g]);
                    const float m_new = fmaxf(m_run[g], tmax);
                    const float pg = (m_new == -INFINITY || sc[g] == -INFINITY) ? 0.f : expf(sc[g] - m_new);
                    const float corr = (m_run[g] == -INFINITY) ? 0.f : expf(m_run[g] - m_new);
                    lsum[g] = fmaf(lsum[g], corr, pg);
                    corr_prev[g] = corr;
                    m_run[g] = m_new;
                    if ((g & 1) == half) {                               // P' column g: one half writes it
                        const float pv = pg * vrs;
                        const uint32_t hb = f16_bits(pv);
                        const uint32_t lb = f16_bits(pv - f16_bits_to_f32(hb));
                        const int kt = t & 63, atom = t >> 6;
                        #pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            const int n = k == 0 ? g : G + g;
                            const uint32_t off = uint32_t(atom * 2048 + (n >> 3) * 1024 + (n & 7) * 128 +
                                                          (((kt >> 3) ^ (n & 7)) << 4) + (kt & 7) * 2);
                            *reinterpret_cast<uint16_t*>(bpv + off) = uint16_t(k == 0 ? hb : lb);
                        }
                    }
                }
                fence_async_smem();
                tc_before();
                mbar_arrive(&M->mb_pvr);                               // V^T and P' written: PV (it)
            }

            // ---- the last tile's PV
            if (!tmo) {
                ewait(&M->mb_pv, ph_pv);
                tc_after();
                if (!tmo) {
                    float pvv[16];
                    tmem_ld16(t_row + PV_COL, pvv);
                    tmem_wait_ld();
                    #pragma unroll
                    for (int g = 0; g < G; ++g) o[g] = fmaf(o[g], corr_prev[g], pvv[g] + pvv[G + g]);
                }
            }
            tmo = epi_any(tmo);
            // softmax denominators: the token sums of half 0's warps (half 1 holds the same)
            if (half == 0) {
                #pragma unroll
                for (int g = 0; g < G; ++g) {
                    float sum = lsum[g];
                    #pragma unroll
                    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                    if (lane == 0) M->red_sum[w][g] = sum;
                }
            }
            epi_sync();
            if (half == 0) {
                #pragma unroll
                for (int g = 0; g < G; ++g) P.part_o[(slot * G + g) * 128 + t] = tmo ? 0.f : o[g];
                if (t < G) {
                    float mt = -INFINITY;
                    #pragma unroll
                    for (int g = 0; g < G; ++g) if (g == t) mt = m_run[g];
                    const float l = M->red_sum[0][t] + M->red_sum[1][t] + M->red_sum[2][t] + M->red_sum[3][t];
                    P.part_ml[(slot * G + t) * 2 + 0] = tmo ? -INFINITY : mt;
                    P.part_ml[(slot * G + t) * 2 + 1] = tmo ? 0.f : l;
                }
            }
            timed_out = tmo;
        }
        // ---- segment end: both roles are done with this segment's shared memory
        timed_out = __syncthreads_or(timed_out);
    }

    // ---- a timeout leaves the rest of the CTA's segments empty
    if (timed_out) {
        while (unit < M->sched_hi && r < P.n_reqs) {
            const int seq = P.seq_lens[r];
            const int nt = req_tiles(seq);
            const int64_t rs = before * nh, re = rs + int64_t(nt) * nh;
            if (unit >= re) { before += nt; ++r; continue; }
            int64_t vs, vs_end;
            share_of(unit, vs, vs_end);
            const int hl = int((unit - rs) / nt);
            const int64_t ps = rs + int64_t(hl) * nt;
            empty_partial(vs + int64_t(r) * nh + hl);
            unit = min(vs_end, ps + nt);
        }
        if (tid == 0) report(P.status, TTKV_STATUS_TIMEOUT);
        // drain: every copy and MMA batch this CTA started gets one more bounded wait (at most one
        // batch of each kind is in flight: the next is issued only after the epilogue has seen the
        // previous one complete)
        if (!epi) {
            asm volatile("cp.async.wait_all;" ::: "memory");
            if (lane == 0) {
                if (n_r) mbar_wait(&M->mb_r, (n_r - 1) & 1u);
                if (n_pv) mbar_wait(&M->mb_pv, (n_pv - 1) & 1u);
                if (pend_dec) mbar_wait(&M->mb_dec, ph_dec);
            }
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    if (w == NEPI / 32) tmem_dealloc(M->tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ host plan
// The shared-memory plan of decode_tw_kernel for a layout, or smem == 0 if it does not fit
// (the quarter-lane kernel then serves it). Two K/V buffers when they fit, else one.
inline TwGeom tw_geom(const ttkv_layout_t* lay, int G) {
    TwGeom T{};
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
    T.kr = std::max(kr, 32);
    T.vr = std::max(vr, 32);
    T.kvrow = T.kr + T.vr;
    if (((T.kvrow >> 4) & 1) == 0) T.kvrow += 16;            // odd 16-byte blocks: no bank conflicts
    const int cch = T.cb >> 4;
    T.cf_swz = (cch % 8 == 0) ? 7 : 0;
    T.cf_pitch = T.cb + ((cch & 1) == 0 && cch % 8 != 0 ? 16 : 0);
    const int atoms = T.natom * ATOM_BYTES;
    const int q_bytes = round_up(G * 128 * 4, 128);
    const int misc = round_up(int(sizeof(TwMisc)), 128);
    for (int nkv = 2; nkv >= 1; --nkv) {
        int off = 0;
        T.off_bhi = off; off += atoms;
        T.off_blo = off; off += atoms;
        T.off_a = off; off += atoms;
        T.off_apv = off; off += APV_BYTES;
        T.off_bpv = off; off += BPV_BYTES;
        T.off_q = off; off += q_bytes;
        T.off_lut = off; off += LUT_BYTES;
        T.off_misc = off; off += misc;
        T.off_bt = off; off += BT_CAP * 4;
        T.off_xs = off; off += 2 * kMaxG * TM * 4;
        T.off_cf = off; off += TM * T.cf_pitch;
        T.off_kv = off; off += nkv * TM * T.kvrow + KV_PAD;
        T.nkv = nkv;
        T.smem = round_up(off, 16) + 1024;
        if (T.smem <= 227 * 1024) return T;
    }
    T.smem = 0;
    return T;
}

}  // namespace tw
