// The decode read on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Included by ttkv_read.cu inside its anonymous namespace (shares ReadParams and the merge).
//
// One CTA = (request, KV head, token split), four warpgroups (512 threads). Token t of the
// current 128-token tile is TMEM lane t; warpgroup c handles a quarter of that token's 128 head
// lanes (the RoPE pairs j, j+64 for j in [16c, 16c+16) of K, the V lanes [32c, 32c+32)). Per tile:
//
//   stage    cp.async (16 B) of each token's coefficient block, this head's K residual row and V
//            row into shared memory, double-buffered across tiles
//   A        coefficients int8 -> fp16 (exact) in the canonical K-major SW128 layout
//   MMA 1    acc[128 tokens x 128 lanes] = A . B_hi + A . B_lo  (fp32 in TMEM), where B is the
//            head's slice of the request's decoder, pre-scaled by a power of two and split into
//            fp16 hi + lo so the product is accurate to ~2^-22 (a single fp16 operand moved
//            attention outputs by 4.4e-4 on the parity store; bf16 by 2.7e-3)
//   decode   while MMA 1 runs: the packed K residual and V codes, eight lanes (one bitmap byte) at a
//            time without branches: a 32-bit window of the code stream at the byte's first code,
//            and per bitmap nibble a table of right shifts that brings each kept lane's code to
//            the bottom (dropped lanes shift by 32 and read 0)
//   epilogue k = acc * (cs * 2^e) + residual; RoPE by the token's own position; partial scores of
//            the G query heads over this warpgroup's lanes, summed across warpgroups in smem;
//            online softmax over the tile by warpgroup 0
//   MMA 2    O^T[128 lanes x 16] = V^T . P', V^T = the tile's V codes (exact small integers in
//            fp16, MN-major so each token writes its lanes contiguously), P' = p * V ruler split
//            into hi (columns 0..G-1) and lo (columns G..2G-1); read back during the next tile
//
// Every wait on an mbarrier is bounded (a clock limit); a timeout sets TTKV_STATUS_TIMEOUT, drains
// what is in flight, frees TMEM and returns. No wait depends on another CTA.

namespace tc {

constexpr int TM = 128;                 // tokens per tile = UMMA M = TMEM lanes
constexpr int NWG = 4;                  // warpgroups; each owns a quarter of every token's lanes
constexpr int NTHR = 128 * NWG;
constexpr uint32_t TMEM_COLS = 256;     // power of two >= 128 (recon) + 16 (PV)
constexpr uint32_t PV_COL = 128;
constexpr int ATOM_BYTES = 128 * 128;   // one SW128 K-major atom column: 128 rows x 128 B
constexpr int APV_BYTES = 32768;        // V^T: 128 tokens x 128 lanes fp16
constexpr int BPV_BYTES = 4096;         // P': 16 rows x 128 tokens fp16
constexpr int LUT_BYTES = 2 * 16 * 16;  // K and V shift tables, 16 nibbles x 4 lanes x u32
constexpr int STAGE_PAD = 16;           // code windows may read up to 7 bytes past a field
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
// Barrier over warpgroup 0 only (named barrier 1).
__device__ __forceinline__ void wg0_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
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

// 8 / 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
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

// ------------------------------------------------------------------ packed fp32 pairs (sm_100)
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// ------------------------------------------------------------------ branch-free code decode
// x >> s with s in [0, 32]; s = 32 gives 0.
__device__ __forceinline__ uint32_t shr_clamp(uint32_t x, uint32_t s) {
    uint32_t d;
    asm("shf.r.clamp.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(0u), "r"(s));
    return d;
}

// Right shift that brings lane k (0..3, MSB-first) of bitmap nibble n to the bottom of a 32-bit
// window whose top holds the nibble's first kept code; 32 (reads 0) for a dropped lane.
__device__ __forceinline__ uint32_t lut_shift(int n, int k, int bits) {
    if (!((n >> (3 - k)) & 1)) return 32u;
    const int before = __popc(n >> (4 - k));                  // kept lanes ahead of k
    return uint32_t(32 - bits * (before + 1));
}

// Bits [bitofs, bitofs + 32) of an MSB-first byte stream in shared memory, first bit at the top.
// `byteoff` is the stream's offset from `sb`; reads the two aligned words holding those 5 bytes.
__device__ __forceinline__ uint32_t window32(const unsigned char* sb, uint32_t byteoff, uint32_t bitofs) {
    const uint32_t b = byteoff + (bitofs >> 3);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(sb + (b & ~3u));
    const uint32_t w0 = wp[0], w1 = wp[1];
    const uint32_t a = (b & 3u) * 0x1111u;
    const uint32_t hi = __byte_perm(w0, w1, 0x0123u + a);     // bytes a..a+3, big-endian
    const uint32_t lo = __byte_perm(w0, w1, 0x4567u + a);     // byte a+4 on top (rest unused)
    return __funnelshift_l(lo, hi, bitofs & 7u);
}

// The four bitmap words of a field that starts `a` bytes into the 32 bytes (x, y): lane l at
// bit 31-(l&31) of word l>>5 (bytes in order, first byte on top). `a` is uniform per CTA.
__device__ __forceinline__ void bitmap_words(uint4 x, uint4 y, int a, uint32_t (&bw)[4]) {
    const uint32_t v[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
    const uint32_t sel = 0x0123u + uint32_t(a & 3) * 0x1111u;
    switch (a >> 2) {
        case 0:
            #pragma unroll
            for (int j = 0; j < 4; ++j) bw[j] = __byte_perm(v[j], v[j + 1], sel);
            break;
        case 1:
            #pragma unroll
            for (int j = 0; j < 4; ++j) bw[j] = __byte_perm(v[j + 1], v[j + 2], sel);
            break;
        case 2:
            #pragma unroll
            for (int j = 0; j < 4; ++j) bw[j] = __byte_perm(v[j + 2], v[j + 3], sel);
            break;
        default:
            #pragma unroll
            for (int j = 0; j < 4; ++j) bw[j] = __byte_perm(v[j + 3], v[j + 4], sel);
            break;
    }
}

// A row keeps at most `kmax` lanes: a malformed bitmap with more set bits drops its highest
// lanes (their codes would lie past the stream), matching the reference's rank < k guard.
__device__ __forceinline__ void trim_bitmap(uint32_t (&bw)[4], int kmax) {
    int excess = __popc(bw[0]) + __popc(bw[1]) + __popc(bw[2]) + __popc(bw[3]) - kmax;
    if (excess <= 0) return;
    #pragma unroll
    for (int j = 3; j >= 0; --j)
        while (excess > 0 && bw[j]) { bw[j] &= bw[j] - 1u; --excess; }
}

// Fields of the 8 lanes of one bitmap byte: `win` = the stream window at the byte's first kept
// code with every code's top bit flipped; f[k] holds lane k's (code ^ 2^(bits-1)) in its low
// `bits` bits, 0 for a dropped lane (higher bits are other codes).
__device__ __forceinline__ void group_fields(uint32_t win, uint32_t byte, int bits, const uint4* lut,
                                             uint32_t (&f)[8]) {
    const uint32_t n0 = byte >> 4, n1 = byte & 15u;
    const uint4 L0 = lut[n0], L1 = lut[n1];
    const uint32_t w1 = win << (uint32_t(bits) * uint32_t(__popc(n0)));
    f[0] = shr_clamp(win, L0.x); f[1] = shr_clamp(win, L0.y);
    f[2] = shr_clamp(win, L0.z); f[3] = shr_clamp(win, L0.w);
    f[4] = shr_clamp(w1, L1.x); f[5] = shr_clamp(w1, L1.y);
    f[6] = shr_clamp(w1, L1.z); f[7] = shr_clamp(w1, L1.w);
}

// Top bits of the 8 code slots of a 32-bit window.
__device__ __forceinline__ uint32_t flip_mask(int bits) {
    uint32_t m = 0;
    #pragma unroll
    for (int s = 0; s < 8; ++s)
        if (bits * (s + 1) <= 32) m |= 1u << (31 - bits * s);
    return m;
}

// Rank of the first lane of bitmap byte `g` (0..15) = set bits in bytes 0..g-1.
__device__ __forceinline__ int byte_rank(const uint32_t (&bw)[4], const int (&pre)[4], int g) {
    const int w = g >> 2, b = g & 3;
    const uint32_t word = w == 0 ? bw[0] : w == 1 ? bw[1] : w == 2 ? bw[2] : bw[3];
    const int p = w == 0 ? pre[0] : w == 1 ? pre[1] : w == 2 ? pre[2] : pre[3];
    return p + (b ? __popc(word >> (32 - 8 * b)) : 0);
}

__device__ __forceinline__ uint32_t bitmap_byte(const uint32_t (&bw)[4], int g) {
    const int w = g >> 2;
    const uint32_t word = w == 0 ? bw[0] : w == 1 ? bw[1] : w == 2 ? bw[2] : bw[3];
    return (word >> (24 - 8 * (g & 3))) & 0xffu;
}

struct TcGeom {            // host-computed shared-memory plan
    int natom, nstage;     // K atoms of 64 ranks; staging buffers
    int kp16;              // r1 rounded up to 16 (the MMA K extent)
    int cb, kr, vr, srow;  // staged bytes per token: coefficient block, K region, V region, total
    int off_bhi, off_blo, off_a, off_apv, off_bpv, off_q, off_red, off_lut, off_misc, off_stage;
    int smem;              // dynamic shared memory requested (includes 1 KB alignment slack)
};

struct TcMisc {
    float red_max[4][kMaxG];
    float red_sum[4][kMaxG];
    float m[kMaxG];
    float l[kMaxG];
    float maxabs[NTHR / 32];
    uint64_t mbar_r, mbar_pv;
    uint32_t tmem_base;
};

template <int G>
__global__ void __launch_bounds__(NTHR, 1) decode_tc_kernel(const ReadParams P, const TcGeom T) {
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    // align inside the shared window by pointer arithmetic, so every access stays a shared access
    unsigned char* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    unsigned char* bhi = base + T.off_bhi;
    unsigned char* blo = base + T.off_blo;
    unsigned char* amat = base + T.off_a;
    unsigned char* apv = base + T.off_apv;
    unsigned char* bpv = base + T.off_bpv;
    float* qs = reinterpret_cast<float*>(base + T.off_q);
    float* red = reinterpret_cast<float*>(base + T.off_red);
    uint4* lutk = reinterpret_cast<uint4*>(base + T.off_lut);
    uint4* lutv = lutk + 16;
    TcMisc* M = reinterpret_cast<TcMisc*>(base + T.off_misc);

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int wg = tid >> 7, t = tid & 127;
    const int split = blockIdx.x, hl = blockIdx.y, r = blockIdx.z;
    const int h = P.head_lo + hl;
    const int seq = P.seq_lens[r];

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
    const int64_t row_base = (int64_t(r) * P.n_heads + hl) * G;
    if (bad || t_begin >= t_end) {
        if (tid < G) {
            P.part_ml[((row_base + tid) * P.n_splits + split) * 2 + 0] = -INFINITY;
            P.part_ml[((row_base + tid) * P.n_splits + split) * 2 + 1] = 0.f;
        }
        if (wg == 0)
            for (int g = 0; g < G; ++g) P.part_o[((row_base + g) * P.n_splits + split) * 128 + t] = 0.f;
        return;
    }

    // ---- set-up: TMEM, barriers, tables, operands that live for the whole CTA
    if (w == 0) tmem_alloc(&M->tmem_base, TMEM_COLS);
    if (tid == 0) { mbar_init(&M->mbar_r, 1); mbar_init(&M->mbar_pv, 1); }
    if (tid < kMaxG) { M->m[tid] = -INFINITY; M->l[tid] = 0.f; }
    if (tid < 32) {
        const int n = tid & 15, bits = tid < 16 ? P.res_bits : P.v_bits;
        (tid < 16 ? lutk : lutv)[n] =
            make_uint4(lut_shift(n, 0, bits), lut_shift(n, 1, bits), lut_shift(n, 2, bits), lut_shift(n, 3, bits));
    }
    for (int i = tid; i < BPV_BYTES / 16; i += NTHR) reinterpret_cast<uint4*>(bpv)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < G * 128; i += NTHR) {
        const int g = i >> 7, j = i & 127;
        qs[i] = load_elt(P.q, P.q_dtype, int64_t(r) * P.q_stride + int64_t(h * G + g) * 128 + j);
    }
    // decoder slice: power-of-two scale so max|D| * 2^-e lies in [2^13, 2^14), then fp16 hi + lo
    const float* dec = P.decoders + int64_t(di) * P.dec_stride + h * 128 + t;
    const int64_t dstride = int64_t(P.H) * 128;
    float mx = 0.f;
    for (int rr = wg; rr < P.r1; rr += NWG) mx = fmaxf(mx, fabsf(dec[rr * dstride]));
    mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
    if (lane == 0) M->maxabs[w] = mx;
    __syncthreads();
    mx = 0.f;
    #pragma unroll
    for (int i = 0; i < NTHR / 32; ++i) mx = fmaxf(mx, M->maxabs[i]);
    int e = 0;
    if (mx > 0.f) e = int((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 13;
    e = max(-100, min(100, e));
    const float s_down = __uint_as_float(uint32_t(127 - e) << 23);   // 2^-e
    const float s_up = __uint_as_float(uint32_t(127 + e) << 23);     // 2^e
    for (int cidx = wg; cidx < T.kp16 / 8; cidx += NWG) {
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

    // ---- staging of one tile: 16-byte chunks of each token's three regions
    const int kfield = P.coeff_bytes + 2 + h * P.k_row;
    const int vfield = P.v_offset + h * P.v_row;
    const int koff = kfield & 15, voff = vfield & 15;
    // chunks this head needs: exactly the 16-byte blocks covering each field, never past the blob
    const int cch = T.cb >> 4;
    const int kch = (koff + P.k_row + 15) >> 4, vch = (voff + P.v_row + 15) >> 4;
    const int nch = cch + kch + vch;
    unsigned char* stage0 = base + T.off_stage;
    auto issue_stage = [&](int t0, unsigned char* st) {
        const int ntok = min(TM, t_end - t0);
        for (int i = tid; i < ntok * nch; i += NTHR) {
            const int tt = i / nch, c = i - tt * nch;
            const int tok = t0 + tt;
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
            cp_async16(st + tt * T.srow + sofs, src + gofs);
        }
        cp_async_commit();
    };

    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t taddr = M->tmem_base;
    const uint32_t t_row = taddr + (uint32_t(32 * (w & 3)) << 16);    // this warp's TMEM lanes

    constexpr uint32_t IDESC_R = idesc_f16(128, 128, false, false);
    constexpr uint32_t IDESC_PV = idesc_f16(128, 16, true, false);
    const int kbits = P.res_bits, vbits = P.v_bits;
    const uint32_t kflip = flip_mask(kbits), vflip = flip_mask(vbits);
    const uint32_t khalf = 1u << (kbits - 1), vhalf = 1u << (vbits - 1);
    const uint32_t kmask = (1u << kbits) - 1u, vmask2 = ((1u << vbits) - 1u) * 0x10001u;
    const uint32_t kmag = 0x4B000000u | khalf;                     // float 2^23 + code
    const float kmag_f = 8388608.f + float(khalf);
    const uint32_t vmag2 = 0x64006400u | (vhalf * 0x10001u);       // fp16 pair 1024 + code
    const __half2 vbias2 = __floats2half2_rn(1024.f + float(vhalf), 1024.f + float(vhalf));
    const bool tbf16 = P.table_dtype == TTKV_BF16;
    const float scale = P.scale;

    float o[G], corr_prev[G];
    #pragma unroll
    for (int g = 0; g < G; ++g) { o[g] = 0.f; corr_prev[g] = 0.f; }
    uint32_t ph_r = 0, ph_pv = 0;
    bool r_pending = false, pv_pending = false, timed_out = false;

    issue_stage(t_begin, stage0);
    int it = 0;
    for (int t0 = t_begin; t0 < t_end; t0 += TM, ++it) {
        unsigned char* st = stage0 + size_t(T.nstage == 2 ? (it & 1) : 0) * (TM * T.srow);
        cp_async_wait_all();
        __syncthreads();                                                   // tile landed
        if (T.nstage == 2 && t0 + TM < t_end)
            issue_stage(t0 + TM, stage0 + size_t((it + 1) & 1) * (TM * T.srow));

        const int tok = t0 + t;
        const bool valid = tok < t_end;
        const unsigned char* srow = st + t * T.srow;
        const uint32_t srow_off = uint32_t(srow - base);

        // ---- A: this token's coefficients as fp16, zero past r1 (and for an invalid token).
        // int8 -> fp16 exactly: flip the sign bit (b + 128 as a byte), place the byte under the
        // fp16 exponent of 1024 (0x64__ = 1024 + byte), subtract 1152.
        for (int c16 = wg; c16 < T.kp16 / 16; c16 += NWG) {
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
            *reinterpret_cast<uint4*>(amat + (cidx >> 3) * ATOM_BYTES + kmajor_off(t, cidx & 7)) =
                make_uint4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<uint4*>(amat + ((cidx + 1) >> 3) * ATOM_BYTES + kmajor_off(t, (cidx + 1) & 7)) =
                make_uint4(hv[4], hv[5], hv[6], hv[7]);
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
            mma_commit(&M->mbar_r);
        }
        r_pending = true;

        // ---- while MMA 1 runs: K residual lanes [16wg, 16wg+16) and [64+16wg, 64+16wg+16)
        const uint32_t kf = srow_off + uint32_t(T.cb + koff);            // K field in smem
        float rkl[16], rkh[16];
        float krs, csp;
        {
            const uint4* kp = reinterpret_cast<const uint4*>(srow + T.cb);
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
            for (int half = 0; half < 2; ++half) {
                #pragma unroll
                for (int gi = 0; gi < 2; ++gi) {
                    const int grp = 8 * half + 2 * wg + gi;
                    const uint32_t byte = bitmap_byte(bw, grp);
                    const int rank = byte_rank(bw, pre, grp);
                    const uint32_t win = window32(base, kf + 16u, uint32_t(rank * kbits)) ^ kflip;
                    uint32_t f[8];
                    group_fields(win, byte, kbits, lutk, f);
                    #pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float v = __uint_as_float((f[k] & kmask) ^ kmag) - kmag_f;
                        if (half == 0) rkl[8 * gi + k] = v; else rkh[8 * gi + k] = v;
                    }
                }
            }
            krs = valid ? f16_at(srow + T.cb + koff + 16 + P.k_pb) : 0.f;
            csp = (valid ? f16_at(srow + P.coeff_bytes) : 0.f) * s_up;
        }

        // ---- PV of the previous tile: fold into o (warpgroup 0), then V^T may be overwritten
        if (pv_pending) {
            if (!mbar_wait(&M->mbar_pv, ph_pv)) timed_out = true;
            else { ph_pv ^= 1u; pv_pending = false; }
            tc_after();
            if (wg == 0 && !__any_sync(0xffffffffu, timed_out)) {
                float d[16];
                tmem_ld16(t_row + PV_COL, d);
                tmem_wait_ld();
                #pragma unroll
                for (int g = 0; g < G; ++g) o[g] = fmaf(o[g], corr_prev[g], d[g] + d[G + g]);
            }
        }

        // ---- V^T (MN-major): lanes [32wg, 32wg+32) of this token as exact small integers
        float vrs;
        {
            const uint32_t vfo = srow_off + uint32_t(T.cb + T.kr + voff);
            const uint4* vp = reinterpret_cast<const uint4*>(srow + T.cb + T.kr);
            uint32_t bw[4];
            bitmap_words(vp[0], vp[1], voff, bw);
            if (!valid) bw[0] = bw[1] = bw[2] = bw[3] = 0u;
            trim_bitmap(bw, P.v_lanes);
            const uint32_t word = wg == 0 ? bw[0] : wg == 1 ? bw[1] : wg == 2 ? bw[2] : bw[3];
            int rank = (wg > 0 ? __popc(bw[0]) : 0) + (wg > 1 ? __popc(bw[1]) : 0) + (wg > 2 ? __popc(bw[2]) : 0);
            #pragma unroll
            for (int gi = 0; gi < 4; ++gi) {
                const uint32_t byte = (word >> (24 - 8 * gi)) & 0xffu;
                const uint32_t win = window32(base, vfo + 16u, uint32_t(rank * vbits)) ^ vflip;
                rank += __popc(byte);
                uint32_t f[8];
                group_fields(win, byte, vbits, lutv, f);
                uint32_t hv[4];
                #pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t x = (__byte_perm(f[2 * k], f[2 * k + 1], 0x5410) & vmask2) ^ vmag2;
                    const __half2 y = __hsub2(*reinterpret_cast<const __half2*>(&x), vbias2);
                    hv[k] = *reinterpret_cast<const uint32_t*>(&y);
                }
                const int ch = 4 * wg + gi;                         // lanes 8ch..8ch+7, one 16-byte chunk
                const uint32_t off = uint32_t((t >> 3) * 2048 + (ch >> 3) * 1024 + (t & 7) * 128 +
                                              (((ch & 7) ^ (t & 7)) << 4));
                *reinterpret_cast<uint4*>(apv + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            }
            vrs = valid ? f16_at(srow + T.cb + T.kr + voff + 16 + P.v_pb) : 0.f;
        }

        // ---- epilogue: rebuild, patch, rotate, partial scores over this warpgroup's lanes
        if (!mbar_wait(&M->mbar_r, ph_r)) timed_out = true;
        else { ph_r ^= 1u; r_pending = false; }
        tc_after();
        float2 s2[G];
        #pragma unroll
        for (int g = 0; g < G; ++g) s2[g] = make_float2(0.f, 0.f);
        if (!__any_sync(0xffffffffu, timed_out)) {
            const uint16_t* trow = reinterpret_cast<const uint16_t*>(P.table) +
                                   int64_t(min(valid ? tok : t_begin, int(P.table_rows - 1))) * 128;
            const float2 csp2 = make_float2(csp, csp), krs2 = make_float2(krs, krs);
            const float2 neg1 = make_float2(-1.f, -1.f);
            #pragma unroll
            for (int hp = 0; hp < 2; ++hp) {                        // 8 RoPE pairs at a time
                const int j0 = 16 * wg + 8 * hp;
                float al[8], ah[8];
                tmem_ld8(t_row + uint32_t(j0), al);
                tmem_ld8(t_row + uint32_t(64 + j0), ah);
                const uint4 cw = __ldg(reinterpret_cast<const uint4*>(trow + j0));
                const uint4 sw = __ldg(reinterpret_cast<const uint4*>(trow + 64 + j0));
                tmem_wait_ld();
                const uint32_t cwv[4] = {cw.x, cw.y, cw.z, cw.w}, swv[4] = {sw.x, sw.y, sw.z, sw.w};
                #pragma unroll
                for (int i = 0; i < 4; ++i) {                       // lanes j0+2i, j0+2i+1
                    float2 cz, sz;
                    if (tbf16) {
                        cz = make_float2(__uint_as_float(cwv[i] << 16), __uint_as_float(cwv[i] & 0xffff0000u));
                        sz = make_float2(__uint_as_float(swv[i] << 16), __uint_as_float(swv[i] & 0xffff0000u));
                    } else {
                        cz = __half22float2(*reinterpret_cast<const __half2*>(&cwv[i]));
                        sz = __half22float2(*reinterpret_cast<const __half2*>(&swv[i]));
                    }
                    const int li = 8 * hp + 2 * i;
                    const float2 kl = f2fma(make_float2(rkl[li], rkl[li + 1]), krs2,
                                            f2mul(make_float2(al[2 * i], al[2 * i + 1]), csp2));
                    const float2 kh = f2fma(make_float2(rkh[li], rkh[li + 1]), krs2,
                                            f2mul(make_float2(ah[2 * i], ah[2 * i + 1]), csp2));
                    const float2 yl = f2fma(f2mul(kh, neg1), sz, f2mul(kl, cz));
                    const float2 yh = f2fma(kl, sz, f2mul(kh, cz));
                    #pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float2 ql = *reinterpret_cast<const float2*>(qs + g * 128 + j0 + 2 * i);
                        const float2 qh = *reinterpret_cast<const float2*>(qs + g * 128 + 64 + j0 + 2 * i);
                        s2[g] = f2fma(ql, yl, f2fma(qh, yh, s2[g]));
                    }
                }
            }
        }
        #pragma unroll
        for (int g = 0; g < G; ++g) red[(wg * G + g) * 128 + t] = s2[g].x + s2[g].y;
        fence_async_smem();                                        // V^T for MMA 2
        if (__syncthreads_or(timed_out)) { timed_out = true; break; }

        // ---- online softmax over the tile (warpgroup 0: thread t = token t)
        if (wg == 0) {
            float sc[G], m_new[G], corr[G];
            #pragma unroll
            for (int g = 0; g < G; ++g) {
                float v = red[g * 128 + t];
                #pragma unroll
                for (int c = 1; c < NWG; ++c) v += red[(c * G + g) * 128 + t];
                sc[g] = valid ? v * scale : -INFINITY;
                float mxg = sc[g];
                #pragma unroll
                for (int off = 16; off; off >>= 1) mxg = fmaxf(mxg, __shfl_xor_sync(0xffffffffu, mxg, off));
                if (lane == 0) M->red_max[w][g] = mxg;
            }
            wg0_sync();
            #pragma unroll
            for (int g = 0; g < G; ++g) {
                const float tmax = fmaxf(fmaxf(M->red_max[0][g], M->red_max[1][g]),
                                         fmaxf(M->red_max[2][g], M->red_max[3][g]));
                const float m_old = M->m[g];
                m_new[g] = fmaxf(m_old, tmax);
                const float pg = (m_new[g] == -INFINITY || sc[g] == -INFINITY) ? 0.f : expf(sc[g] - m_new[g]);
                corr[g] = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new[g]);
                float sum = pg;
                #pragma unroll
                for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                if (lane == 0) M->red_sum[w][g] = sum;
                // P' = p * V ruler as fp16 hi (column g) + lo (column G + g); this token is K index t
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
            wg0_sync();
            if (t < G) {
                #pragma unroll
                for (int g = 0; g < G; ++g) {
                    if (t == g) {
                        const float tsum = M->red_sum[0][g] + M->red_sum[1][g] + M->red_sum[2][g] + M->red_sum[3][g];
                        M->l[g] = M->l[g] * corr[g] + tsum;
                        M->m[g] = m_new[g];
                    }
                }
            }
            #pragma unroll
            for (int g = 0; g < G; ++g) corr_prev[g] = corr[g];
        }
        fence_async_smem();
        tc_before();
        __syncthreads();
        tc_after();

        // ---- MMA 2: O^T[lane][col] = V^T . P'  (8 K-steps of 16 tokens); read in the next tile
        if (tid == 0) {
            const uint32_t a0 = smem_u32(apv), b0 = smem_u32(bpv);
            for (int ks = 0; ks < TM / 16; ++ks) {
                const uint64_t ad = sw128_desc(a0 + uint32_t(ks * 4096), 1024, 2048);
                const uint64_t bd = sw128_desc(b0 + uint32_t((ks >> 2) * 2048 + (ks & 3) * 32), 16, 1024);
                mma_f16(taddr + PV_COL, ad, bd, IDESC_PV, ks > 0 ? 1u : 0u);
            }
            mma_commit(&M->mbar_pv);
        }
        pv_pending = true;
        if (T.nstage == 1 && t0 + TM < t_end) issue_stage(t0 + TM, stage0);   // every read of the stage is done
    }

    // ---- the last tile's PV
    if (!timed_out && pv_pending) {
        if (!mbar_wait(&M->mbar_pv, ph_pv)) timed_out = true;
        else { ph_pv ^= 1u; pv_pending = false; }
        tc_after();
        if (wg == 0 && !__any_sync(0xffffffffu, timed_out)) {
            float d[16];
            tmem_ld16(t_row + PV_COL, d);
            tmem_wait_ld();
            #pragma unroll
            for (int g = 0; g < G; ++g) o[g] = fmaf(o[g], corr_prev[g], d[g] + d[G + g]);
        }
    }
    timed_out = __syncthreads_or(timed_out);

    // ---- drain and release: anything still in flight gets one more bounded wait before TMEM is freed
    if (timed_out) {
        if (tid == 0) report(P.status, TTKV_STATUS_TIMEOUT);
        if (r_pending) mbar_wait(&M->mbar_r, ph_r);
        if (pv_pending) mbar_wait(&M->mbar_pv, ph_pv);
    }
    cp_async_wait_all();
    tc_before();
    __syncthreads();
    tc_after();
    if (w == 0) tmem_dealloc(taddr, TMEM_COLS);
    if (wg == 0) {
        #pragma unroll
        for (int g = 0; g < G; ++g)
            P.part_o[((row_base + g) * P.n_splits + split) * 128 + t] = timed_out ? 0.f : o[g];
    }
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
    // the bitmap is read as the two 16-byte chunks holding it
    T.kr = std::max(kr, 32);
    T.vr = std::max(vr, 32);
    T.srow = T.cb + T.kr + T.vr;
    const int atoms = T.natom * ATOM_BYTES;
    const int q_bytes = round_up(G * 128 * 4, 1024);
    const int red_bytes = round_up(NWG * G * 128 * 4, 1024);
    const int misc = round_up(int(sizeof(TcMisc)), 128);
    for (int ns = 2; ns >= 1; --ns) {
        int off = 0;
        T.off_bhi = off; off += atoms;
        T.off_blo = off; off += atoms;
        T.off_a = off; off += atoms;
        T.off_apv = off; off += APV_BYTES;
        T.off_bpv = off; off += BPV_BYTES;
        T.off_q = off; off += q_bytes;
        T.off_red = off; off += red_bytes;
        T.off_lut = off; off += LUT_BYTES;
        T.off_misc = off; off += misc;
        T.off_stage = off; off += ns * TM * T.srow + STAGE_PAD;
        T.nstage = ns;
        T.smem = off + 1024;
        if (T.smem <= 227 * 1024) return T;
    }
    T.smem = 0;
    return T;
}

}  // namespace tc
