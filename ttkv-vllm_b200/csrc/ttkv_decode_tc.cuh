// The decode read on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Included by ttkv_read.cu inside its anonymous namespace (shares ReadParams and the merge).
//
// The launch is one CTA per SM, four warpgroups (512 threads) each, whatever the batch's lengths.
// The work is the list of (request, KV head, 128-token tile) units, request-major; CTA c takes the
// c-th equal share of it, computed on the device from seq_lens, and walks it as segments, one per
// (request, KV head) it touches, each leaving a partial (o, max, sum) that merge_sk_kernel
// combines. A segment spans at most BT_CAP blocks (the bound the workspace is sized with), so when
// the shares would be longer than that the device cuts every share into k equal virtual shares
// (k from the batch's total), and a segment also ends at a virtual boundary. Within a segment, token t of the current tile is TMEM lane t;
// warpgroup c handles a quarter of that token's 128 head lanes (the RoPE pairs j, j+64 for j in
// [16c, 16c+16) of K, the V lanes [32c, 32c+32)). Per tile:
//
//   stage    16-byte cp.async copies, chunk-fastest over the tile's tokens, completing on an
//            mbarrier per unit: this head's K and V rows (two buffers, two tiles ahead), the
//            coefficient block (one buffer, one tile ahead of its conversion) and the RoPE row
//            (one buffer, rows padded to 272 B)
//   A        coefficients int8 -> fp16 (exact) in the canonical K-major SW128 layout, converted
//            for the next tile as soon as this tile's MMA 1 has read A
//   MMA 1    acc[128 tokens x 128 lanes] = A . B_hi + A . B_lo  (fp32 in TMEM, two column sets
//            so the next tile's MMA runs under this tile's softmax), where B is the head's slice
//            of the request's decoder, pre-scaled by a power of two and split into fp16 hi + lo so
//            the product is accurate to ~2^-22 (a single fp16 operand moved attention outputs by
//            4.4e-4 on the parity store; bf16 by 2.7e-3)
//   decode   the packed K residual and V codes, eight lanes (one bitmap byte) at a time without
//            branches: a 32-bit window of the code stream at the byte's first code, and per bitmap
//            nibble a table of right shifts that brings each kept lane's code to the bottom
//            (dropped lanes shift by 32 and read 0)
//   epilogue k = acc * (cs * 2^e) + residual; RoPE by the token's own position; partial scores of
//            the G query heads over this warpgroup's lanes, summed across warpgroups through
//            TMEM; online softmax over the tile, warpgroup g owning query head g
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
constexpr uint32_t TMEM_COLS = 512;     // 2 x 128 (recon, double-buffered) + 16 (PV) + 32 (partial scores)
constexpr uint32_t PV_COL = 256;
constexpr int ATOM_BYTES = 128 * 128;   // one SW128 K-major atom column: 128 rows x 128 B
constexpr int APV_BYTES = 32768;        // V^T: 128 tokens x 128 lanes fp16
constexpr int BPV_BYTES = 4096;         // P': 16 rows x 128 tokens fp16
constexpr int LUT_BYTES = 2 * 16 * 16;  // K and V shift tables, 16 nibbles x 4 lanes x u32
constexpr int STAGE_PAD = 16;           // code windows may read up to 7 bytes past a field

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


// Byte offset of (row, 16-byte chunk) in a K-major SW128 atom column of 128-byte rows.
__device__ __forceinline__ uint32_t kmajor_off(int row, int chunk) {
    return uint32_t((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------------ packed fp32 pairs (sm_100)
// The compiler's own f32x2 builtins: it places the pairs in adjacent registers itself and can
// fold a negated operand, which an asm block that packs its operands with mov.b64 cannot.
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) { return __fmul2_rn(a, b); }

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
    int natom;             // K atoms of 64 ranks
    int kp16;              // r1 rounded up to 16 (the MMA K extent)
    int cb, cf_pitch;      // staged coefficient block per token (coefficients + scale, 16-byte
                           // blocks) and its row pitch in shared memory
    int cf_swz;            // 7: 16-byte block c of token u is stored at block c ^ (u & 7)
    int kr, vr, kvrow;     // staged K region, V region, and the row pitch of both
    int nkv;               // K/V staging buffers (2: filled a tile ahead; 1: after the tile's reads)
    int rope_smem;         // 1: the tile's RoPE rows are staged in shared memory
    int off_bhi, off_blo, off_a, off_apv, off_bpv, off_q, off_lut, off_misc, off_bt, off_cf, off_kv, off_rp;
    int smem;              // dynamic shared memory requested (includes 1 KB alignment slack)
};

// The TMA map of a launch's RoPE table: boxes of 128 rows x 64 values (the cos or the sin half).
struct TcMaps {
    CUtensorMap rope;
};

constexpr int RP_BOX = 128 * 128;        // one TMA box of RoPE rows: 128 positions x 64 x 16-bit
constexpr int BT_CAP = 512;              // blocks a segment may span; its shared region (2 KB) holds
                                         // the slot-row offsets of two tiles
constexpr int KV_PAD = 16;               // code windows may read a few bytes past the last row
constexpr uint32_t RED_COL = 272;        // TMEM columns of the partial scores: [warpgroup][8 heads]

struct TcMisc {
    float red_max[4][kMaxG];
    float red_sum[4][kMaxG];
    float m[kMaxG];
    float l[kMaxG];
    float maxabs[NTHR / 32];
    int scan[NTHR / 32];
    int sched_r;
    long long sched_before;
    long long sched_T, sched_nv, sched_hi;   // the batch's units, virtual shares, this CTA's end
    long long seg_slot;                      // the current segment's partial slot
    int lim[kMaxG];                          // row g sees the segment's rows before lim[g]
    uint64_t mb_r, mb_pv, mb_cf, mb_rp, mb_kv[2], mb_dec;
    uint32_t tmem_base;
};

// Query heads whose softmax a warpgroup owns: g = wg + NWG * i, i < HPW.
constexpr int HPW = (kMaxG + NWG - 1) / NWG;
constexpr int MMA_TID = NTHR - 32;       // lane 0 of the last warp issues every MMA
constexpr int MAX_R1 = 192;              // largest r1 the tensor-core decode serves
constexpr int DEC_CHUNKS = (MAX_R1 / 8 + NWG - 1) / NWG;   // 8-row decoder chunks per warpgroup
constexpr int RP_TID = NTHR - 64;        // lane 0 of the warp before it issues the RoPE loads

// Max over the warp (sm_100a redux on fp32).
__device__ __forceinline__ float warp_max(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// Named barrier over the 128 threads of warpgroup `wg` (ids 1..4; 0 is __syncthreads).
__device__ __forceinline__ void wg_sync(int wg) {
    asm volatile("bar.sync %0, 128;" :: "r"(wg + 1) : "memory");
}

__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
    return __uint_as_float(r);
}

// 8 consecutive fp32 columns of this thread's TMEM lane (then tcgen05.wait::st before a barrier).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
        :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
           "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
           "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Tiles of a request (a request with no rows has none).
__device__ __forceinline__ int req_tiles(int seq) { return seq > 0 ? (seq + TM - 1) / TM : 0; }

// Tiles a segment may span so that its tokens stay within BT_CAP blocks of `block_size` (a run of
// s tiles starting at a tile boundary touches at most s*TM/block_size + 1 blocks).
__host__ __device__ __forceinline__ int64_t share_cap(int block_size) {
    const int64_t c = int64_t(BT_CAP - 1) * block_size / TM;
    return c > 0 ? c : 1;
}

// k: the virtual shares per CTA, the least that keeps every share of T units over n CTAs within
// share_cap tiles (a share of T / (n k) units holds at most ceil of that).
__host__ __device__ __forceinline__ int64_t virtual_shares(int64_t T, int64_t n, int block_size) {
    const int64_t per = n * share_cap(block_size);
    return T > per ? (T + per - 1) / per : 1;
}

// Exclusive prefix sum of v over the CTA's threads in thread order, and the CTA's total. Every
// thread of the CTA calls it; `wsum` is NTHR / 32 ints of shared memory.
__device__ __forceinline__ int cta_scan(int v, int* wsum, int& total) {
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
    for (int i = 0; i < NTHR / 32; ++i) {
        const int sw = wsum[i];
        if (i < w) pre += sw;
        total += sw;
    }
    __syncthreads();
    return pre + x - v;
}

// TBF16: the RoPE table holds bf16 (else fp16) values, fixed at compile time so the conversion of
// its rows costs no per-element select
template <int G, bool TBF16>
__global__ void __launch_bounds__(NTHR, 1) decode_tc_kernel(const ReadParams P, const TcGeom T,
                                                             const __grid_constant__ TcMaps maps) {
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    // align inside the shared window by pointer arithmetic, so every access stays a shared access
    unsigned char* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
    unsigned char* bhi = base + T.off_bhi;
    unsigned char* blo = base + T.off_blo;
    unsigned char* amat = base + T.off_a;
    unsigned char* apv = base + T.off_apv;
    unsigned char* bpv = base + T.off_bpv;
    float* qs = reinterpret_cast<float*>(base + T.off_q);        // [g][pair i2][q_2i2, q_2i2+1, q_64+2i2, q_65+2i2]
    uint4* lutk = reinterpret_cast<uint4*>(base + T.off_lut);
    uint4* lutv = lutk + 16;
    TcMisc* M = reinterpret_cast<TcMisc*>(base + T.off_misc);
    unsigned char* cfb = base + T.off_cf;                         // [token][cf_pitch]
    unsigned char* kvb = base + T.off_kv;                         // [buffer][token][K region | V region]
    unsigned char* rpb = base + T.off_rp;                         // [cos | sin][token][128 B], SW128

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int wg = tid >> 7, t = tid & 127;
    const int nh = P.n_heads;
    // launched while the kernel before it may still run: everything this kernel reads (seq_lens,
    // the block table, q, the decoders, the cache) may come from that kernel
    pdl_wait();

    // ---- the schedule. Units are (request, KV head, 128-token tile) in request-major order;
    // T = n_heads * sum over requests of their tiles, from the device's seq_lens. CTA c takes the
    // units [c*T/n, (c+1)*T/n) of the n CTAs, so every SM gets the same amount of work whatever
    // the batch's lengths; a run that crosses a (request, head) boundary is processed as one
    // segment per pair, each leaving a partial (o, max, sum) for the merge.
    int64_t T_units, lo, hi;
    int r = 0;
    int64_t before = 0;
    if (P.n_reqs <= NTHR) {                       // one pass: thread i holds request i
        const int v = tid < P.n_reqs ? req_tiles(P.seq_lens[tid]) : 0;
        int tot;
        const int ex = cta_scan(v, M->scan, tot);
        T_units = int64_t(tot) * nh;
        lo = int64_t(blockIdx.x) * T_units / gridDim.x;
        hi = int64_t(blockIdx.x + 1) * T_units / gridDim.x;
        if (tid < P.n_reqs && int64_t(ex) * nh <= lo && lo < int64_t(ex + v) * nh) {
            M->sched_r = tid;
            M->sched_before = ex;
        }
    } else {                                      // the total first, then the request holding lo
        int64_t tiles_all = 0;
        for (int base0 = 0; base0 < P.n_reqs; base0 += NTHR) {
            const int i = base0 + tid;
            int tot;
            cta_scan(i < P.n_reqs ? req_tiles(P.seq_lens[i]) : 0, M->scan, tot);
            tiles_all += tot;
        }
        T_units = tiles_all * nh;
        lo = int64_t(blockIdx.x) * T_units / gridDim.x;
        hi = int64_t(blockIdx.x + 1) * T_units / gridDim.x;
        int64_t acc = 0;
        for (int base0 = 0; base0 < P.n_reqs && acc * nh <= lo; base0 += NTHR) {
            const int i = base0 + tid;
            const int v = i < P.n_reqs ? req_tiles(P.seq_lens[i]) : 0;
            int tot;
            const int ex = cta_scan(v, M->scan, tot);
            if (i < P.n_reqs && (acc + ex) * nh <= lo && lo < (acc + ex + v) * nh) {
                M->sched_r = i;
                M->sched_before = acc + ex;
            }
            acc += tot;                                        // uniform: the CTA's sum
        }
    }
    // virtual shares: nv = gridDim.x * k equal shares of T, k the least that keeps a share within
    // `cap` tiles; CTA c walks shares c*k .. c*k + k - 1 (its range [lo, hi) is their union). Kept
    // in shared memory and read per segment, which saves their registers for the tile loop.
    const int64_t nv = int64_t(gridDim.x) * virtual_shares(T_units, gridDim.x, P.block_size);
    if (tid == 0) { M->sched_T = T_units; M->sched_nv = nv; M->sched_hi = hi; }
    __syncthreads();
    pdl_trigger();                                             // the merge may launch
    if (nv + int64_t(P.n_reqs) * nh > P.n_part_slots) {       // uniform: seq_lens above the bound
        if (blockIdx.x == 0 && tid == 0) report(P.status, TTKV_STATUS_SEQ_BOUND);
        return;
    }
    if (lo >= hi) return;                                      // uniform: nothing for this CTA
    r = M->sched_r;
    before = M->sched_before;
    int64_t unit = lo;
    // the virtual share holding unit u: v = ceil((u + 1) nv / T) - 1; it ends at (v + 1) T / nv
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
        if (wg == 0)
            for (int g = 0; g < G; ++g) P.part_o[(slot * G + g) * 128 + t] = 0.f;
    };

    // ---- set-up for the CTA's lifetime: TMEM, barriers, shift tables, the zero columns of P'
    if (w == 0) tmem_alloc(&M->tmem_base, TMEM_COLS);
    if (tid == RP_TID && T.rope_smem) tma_prefetch_desc(&maps.rope);
    if (tid == 0) {
        mbar_init(&M->mb_r, 1);
        mbar_init(&M->mb_pv, 1);
        mbar_init(&M->mb_cf, NTHR);
        mbar_init(&M->mb_rp, 1);
        mbar_init(&M->mb_kv[0], NTHR);
        mbar_init(&M->mb_kv[1], NTHR);
        mbar_init(&M->mb_dec, 1);
    }
    if (tid < 32) {
        const int n = tid & 15, bits = tid < 16 ? P.res_bits : P.v_bits;
        (tid < 16 ? lutk : lutv)[n] =
            make_uint4(lut_shift(n, 0, bits), lut_shift(n, 1, bits), lut_shift(n, 2, bits), lut_shift(n, 3, bits));
    }
    for (int i = tid; i < BPV_BYTES / 16; i += NTHR) reinterpret_cast<uint4*>(bpv)[i] = make_uint4(0, 0, 0, 0);

    auto kv_buf = [&](int tile) { return T.nkv == 2 ? (tile & 1) : 0; };
    // phase parities of the staging mbarriers, and which have copies in flight
    uint32_t par_cf = 0, par_rp = 0, par_kv0 = 0, par_kv1 = 0;
    bool pend_cf = false, pend_rp = false, pend_kv0 = false, pend_kv1 = false;
    bool timed_out = false;
    auto wait_cf = [&]() {
        if (!mbar_wait(&M->mb_cf, par_cf)) timed_out = true; else { par_cf ^= 1u; pend_cf = false; }
    };
    auto wait_rp = [&]() {
        if (!mbar_wait(&M->mb_rp, par_rp)) timed_out = true; else { par_rp ^= 1u; pend_rp = false; }
    };
    auto wait_kv = [&](int b) {
        if (!mbar_wait(&M->mb_kv[b], b ? par_kv1 : par_kv0)) timed_out = true;
        else if (b) { par_kv1 ^= 1u; pend_kv1 = false; }
        else { par_kv0 ^= 1u; pend_kv0 = false; }
    };
    auto mark_kv = [&](int tile) { if (kv_buf(tile)) pend_kv1 = true; else pend_kv0 = true; };

    // ---- A: a token's coefficients as fp16 (16 per chunk, chunks wg, wg + NWG, ...), zero past r1
    // and for an invalid token. int8 -> fp16 exactly: flip the sign bit (b + 128 as a byte), place
    // the byte under the fp16 exponent of 1024 (0x64__ = 1024 + byte), subtract 1152.
    auto convert_a = [&](bool valid) {
        const unsigned char* srow = cfb + t * T.cf_pitch;
        const int swz = t & T.cf_swz;
        for (int c16 = wg; c16 < T.kp16 / 16; c16 += NWG) {
            uint4 raw = valid ? *reinterpret_cast<const uint4*>(srow + 16 * (c16 ^ swz)) : make_uint4(0, 0, 0, 0);
            const int left = P.r1 - 16 * c16;                       // coefficient bytes in this chunk
            uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
            if (left < 16) {
                #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int keep = left - 4 * i;                  // bytes of this word that are coefficients
                    const uint32_t mask = keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : (0xffffffffu >> (8 * (4 - keep)));
                    wds[i] &= mask;
                }
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
        // the token's coefficient scale: fp16 at bytes coeff_bytes, +1 (they may sit in two blocks)
        auto byte_at = [&](int b) { return uint32_t(srow[16 * ((b >> 4) ^ swz) + (b & 15)]); };
        const int sb = P.coeff_bytes;
        return valid ? f16_bits_to_f32(byte_at(sb) | (byte_at(sb + 1) << 8)) : 0.f;
    };

    // MMA issue (one thread). The start-address field of a descriptor is its low 14 bits (16-byte
    // units, shared addresses < 2^18 B), so a k-step offset is added to the descriptor directly.
    const uint64_t dA = sw128_desc(smem_u32(amat), 16, 1024), dH = sw128_desc(smem_u32(bhi), 16, 1024),
                   dL = sw128_desc(smem_u32(blo), 16, 1024);
    const uint64_t dV = sw128_desc(smem_u32(apv), 1024, 2048), dP = sw128_desc(smem_u32(bpv), 16, 1024);
    auto issue_recon = [&](uint32_t d_tmem) {
        constexpr uint32_t IDESC_R = idesc_f16(128, 128, false, false);
        for (int ks = 0; ks < T.kp16 / 16; ++ks) {
            const uint64_t k16 = uint64_t(((ks >> 2) * ATOM_BYTES + (ks & 3) * 32) >> 4);
            mma_f16(d_tmem, dA + k16, dH + k16, IDESC_R, ks > 0 ? 1u : 0u);
            mma_f16(d_tmem, dA + k16, dL + k16, IDESC_R, 1u);
        }
        mma_commit(&M->mb_r);
    };
    auto issue_pv = [&](uint32_t d_tmem) {
        constexpr uint32_t IDESC_PV = idesc_f16(128, 16, true, false);
        #pragma unroll
        for (int ks = 0; ks < TM / 16; ++ks)
            mma_f16(d_tmem, dV + uint64_t((ks * 4096) >> 4),
                    dP + uint64_t(((ks >> 2) * 2048 + (ks & 3) * 32) >> 4), IDESC_PV, ks > 0 ? 1u : 0u);
        mma_commit(&M->mb_pv);
    };

    const int kbits = P.res_bits, vbits = P.v_bits;
    const uint32_t kflip = flip_mask(kbits), vflip = flip_mask(vbits);
    const uint32_t khalf = 1u << (kbits - 1), vhalf = 1u << (vbits - 1);
    const uint32_t kmask = (1u << kbits) - 1u, vmask2 = ((1u << vbits) - 1u) * 0x10001u;
    const uint32_t kmag = 0x4B000000u | khalf;                     // float 2^23 + code
    const float kmag_f = 8388608.f + float(khalf);
    const uint32_t vmag2 = 0x64006400u | (vhalf * 0x10001u);       // fp16 pair 1024 + code
    const __half2 vbias2 = __floats2half2_rn(1024.f + float(vhalf), 1024.f + float(vhalf));
    constexpr bool tbf16 = TBF16;
    const float scale = P.scale;
    const float4* qs4 = reinterpret_cast<const float4*>(qs);

    uint32_t ph_r = 0, ph_pv = 0, ph_dec = 0;
    bool r_pending_any = false, pv_pending_any = false, pend_dec = false;

    while (unit < M->sched_hi && !timed_out) {
        // ---- the next segment: the run of this CTA's units that belongs to one (request, KV head)
        if (r >= P.n_reqs) break;                                   // unreachable: hi <= T
        // the segment's two scalar loads go out together (a continuation launch's request r is a
        // block of queries of stored request rq)
        const int seq = P.seq_lens[r];
        const int rq = P.v_req ? P.v_req[r] : r;
        const int di = P.dec_index[rq];
        const int nt = req_tiles(seq);
        const int64_t rs = before * nh, re = rs + int64_t(nt) * nh;
        if (unit >= re) { before += nt; ++r; continue; }        // past this request (or it has no rows)
        int64_t vs, vs_end;
        share_of(unit, vs, vs_end);
        const int hl = int((unit - rs) / nt);
        const int64_t ps = rs + int64_t(hl) * nt;
        const int64_t seg_hi = min(vs_end, ps + nt);                // vs_end <= the CTA's end
        const int t_begin = int(unit - ps) * TM;
        const int t_end = min(seq, int(seg_hi - ps) * TM);
        const int64_t slot = vs + int64_t(r) * nh + hl;
        if (tid == 0) M->seg_slot = slot;       // read again at the segment's end (registers)
        unit = seg_hi;
        const int h = P.head_lo + hl;

        // ---- the cheap refusals (uniform); the block ids are checked as the set-up loads them
        bool bad = false;
        if (seq > P.max_seq) { if (tid == 0) report(P.status, TTKV_STATUS_SEQ_BOUND); bad = true; }
        if (!bad && (di < 0 || di >= P.n_decoders)) { if (tid == 0) report(P.status, TTKV_STATUS_DECODER); bad = true; }
        const int blocks_needed = (seq + P.block_size - 1) / P.block_size;
        if (!bad && blocks_needed > P.bt_cols) { if (tid == 0) report(P.status, TTKV_STATUS_ROW_SHORT); bad = true; }
        const int32_t* brow = P.block_table + int64_t(rq) * P.bt_stride;
        if (!bad && (t_end - 1) / P.block_size - t_begin / P.block_size + 1 > BT_CAP) {
            if (tid == 0) report(P.status, TTKV_STATUS_ROW_SHORT);   // the plan keeps a segment within BT_CAP blocks
            bad = true;
        }
        const int n_tiles = (t_end - t_begin + TM - 1) / TM;

        // ---- staging. Per tile, 16-byte cp.async copies laid out chunk-fastest over the tile's tokens
        // (a warp's copies cover a few consecutive slot fields, not 32 scattered rows), the issue cost
        // shared by every warp: the coefficient blocks (one buffer, refilled after the softmax
        // barrier for the tile after next) and this head's K and V fields (T.nkv buffers, refilled at
        // the top of the tile before), each field exactly the 16-byte blocks covering it, never past
        // the blob. Every thread arrives once per phase on the unit's mbarrier after its own copies
        // (cp.async.mbarrier.arrive.noinc). The tile's RoPE rows are consecutive positions of the
        // table: two TMA boxes (cos, sin) of 128 rows, 128-byte swizzled, from one thread.
        const int kfield = P.coeff_bytes + 2 + h * P.k_row;
        const int vfield = P.v_offset + h * P.v_row;
        const int koff = kfield & 15, voff = vfield & 15;
        const int cch = T.cb >> 4;
        const int kch = (koff + P.k_row + 15) >> 4, vch = (voff + P.v_row + 15) >> 4;
        const int nkvc = kch + vch;
        // division by the chunk counts and the block size as a multiply-high (operands < 2^32 / divisor)
        const uint32_t mul_cf = uint32_t((0x100000000ull + cch - 1) / cch);
        const uint32_t mul_kv = uint32_t((0x100000000ull + nkvc - 1) / nkvc);
        const uint32_t bsz = uint32_t(P.block_size);
        const uint64_t mul_bs = (0x100000000ull + bsz - 1) / bsz;
        const int blk0 = t_begin / P.block_size;
        static_assert(BT_CAP * 4 >= 2 * TM * 8, "the slot-row table lives in the block-table region");
        auto slot_at = [&](int tok) -> int64_t {              // tok of this segment (its blocks are checked)
            const uint32_t blk = uint32_t((uint64_t(uint32_t(tok)) * mul_bs) >> 32);
            return int64_t(brow[blk]) * P.block_size + int64_t(uint32_t(tok) - blk * bsz);
        };
        auto ntok = [&](int tile) { return tile < n_tiles ? min(TM, t_end - (t_begin + tile * TM)) : 0; };
        // byte offsets of the slot rows of a tile's tokens (slot * row_bytes), two tiles' worth by
        // tile parity, written one barrier before the copies of that tile go out, so that a copy
        // costs one shared load instead of a block lookup
        int64_t* trs = reinterpret_cast<int64_t*>(base + T.off_bt);
        auto fill_rows = [&](int tile, int u) {
            trs[(tile & 1) * TM + u] = u < ntok(tile) ? slot_at(t_begin + tile * TM + u) * P.row_bytes : 0;
        };
        auto issue_cf = [&](int tile) {
            const int n = ntok(tile) * cch;
            const int64_t* tr = trs + (tile & 1) * TM;
            for (int i = tid; i < n; i += NTHR) {
                // i / cch as a multiply-high; a one-chunk block (r1 <= 14) has no such multiplier
                const uint32_t u = cch == 1 ? uint32_t(i) : __umulhi(uint32_t(i), mul_cf),
                               c = uint32_t(i) - u * uint32_t(cch);
                cp_async16(cfb + u * T.cf_pitch + 16 * (c ^ (u & uint32_t(T.cf_swz))), P.cache + tr[u] + 16 * c);
            }
            cp_async_arrive(&M->mb_cf);
        };
        auto issue_kv = [&](int tile) {
            const int b = kv_buf(tile), n = ntok(tile) * nkvc;
            const int64_t* tr = trs + (tile & 1) * TM;
            unsigned char* dstb = kvb + size_t(b) * TM * T.kvrow;
            for (int i = tid; i < n; i += NTHR) {
                const uint32_t u = __umulhi(uint32_t(i), mul_kv), c = uint32_t(i) - u * uint32_t(nkvc);
                const uint8_t* src = P.cache + tr[u];
                unsigned char* dst = dstb + u * T.kvrow;
                if (int(c) < kch) cp_async16(dst + 16 * c, src + (kfield - koff) + 16 * c);
                else cp_async16(dst + T.kr + 16 * (c - kch), src + (vfield - voff) + 16 * (c - kch));
            }
            cp_async_arrive(&M->mb_kv[b]);
        };
        auto issue_rp = [&](int tile) {                                // RP_TID only; the buffer is free
            mbar_expect_tx(&M->mb_rp, uint32_t(2 * RP_BOX));
            tma_load_2d(rpb, &maps.rope, 0, t_begin + tile * TM, &M->mb_rp);
            tma_load_2d(rpb + RP_BOX, &maps.rope, 64, t_begin + tile * TM, &M->mb_rp);
        };
        // ---- the segment's set-up. Pass 1: its block ids (each checked against the cache) and
        // its query rows; then the slot rows of its first two tiles and the first tile's copies. Pass 2, under
        // those copies: the largest |value| of its decoder slice, coalesced rows w + 16 i. After
        // that barrier thread t converts column t of the 8-row chunks wg, wg + NWG, ...
        const float* dec = P.decoders + int64_t(bad ? 0 : di) * P.dec_stride + h * 128 + t;
        const int64_t dstride = int64_t(P.H) * 128;
        const int nchunk = T.kp16 / 8;
        int local_bad = 0;
        if (!bad) {
            // one pass with every load issued before any is used: this thread's block id of the
            // segment (nblk <= BT_CAP = NTHR), the block of its token of the first two tiles (for
            // their slot-row tables), and its query values (G * 128 <= 2 NTHR)
            static_assert(BT_CAP <= NTHR && kMaxG * 128 <= 2 * NTHR, "one pass of the set-up");
            const int nblk = (t_end - 1) / P.block_size - blk0 + 1;        // <= BT_CAP (checked above)
            const int64_t n_blocks = P.n_slots / P.block_size;
            const int32_t blk = tid < nblk ? brow[blk0 + tid] : 0;
            const int ft = tid >> 7, fu = tid & 127;
            const bool frow = tid < 2 * TM && fu < ntok(ft);            // ntok is 0 past the last tile
            const int ftok = t_begin + ft * TM + fu;
            const uint32_t fb = frow ? uint32_t((uint64_t(uint32_t(ftok)) * mul_bs) >> 32) : 0u;
            const int32_t fblk = frow ? brow[fb] : 0;
            float qv[2];
            int qi[2];
            #pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int i = tid + k * NTHR;
                const int g = i >> 7, j = i & 127;
                qi[k] = i < G * 128 ? (g * 32 + ((j & 63) >> 1)) * 4 + (j >= 64 ? 2 : 0) + (j & 1) : -1;
                qv[k] = 0.f;
                if (i < G * 128) {
                    if (!P.v_req) {
                        qv[k] = load_elt(P.q, P.q_dtype, int64_t(r) * P.q_stride + int64_t(h * G + g) * 128 + j);
                    } else if (g < P.v_nq[r]) {          // row g = (query jq, head gh) of the block
                        const int f = P.v_f0[r] + g, jq = f / P.g_real, gh = f - jq * P.g_real;
                        qv[k] = load_elt(P.q, P.q_dtype, int64_t(P.v_qrow[r] + jq) * P.q_stride +
                                                         int64_t(h * P.g_real + gh) * 128 + j);
                    }
                }
            }
            if (tid < nblk && (blk < 0 || blk >= n_blocks)) local_bad = 1;
            // the first two tiles' slot rows (a bad block id makes the segment skipped: unused)
            if (tid < 2 * TM)
                trs[(ft & 1) * TM + fu] = frow ? (int64_t(fblk) * P.block_size + int64_t(uint32_t(ftok) - fb * bsz)) * P.row_bytes : 0;
            #pragma unroll
            for (int k = 0; k < 2; ++k)
                if (qi[k] >= 0) qs[qi[k]] = qv[k];
        }
        if (tid < kMaxG) {
            M->m[tid] = -INFINITY;
            M->l[tid] = 0.f;
            // causal rows of a continuation block: query jq sees positions <= v_pos + jq
            int lim = 0x7fffffff;
            if (P.v_req) lim = tid < P.v_nq[r] ? P.v_pos[r] + (P.v_f0[r] + tid) / P.g_real + 1 : 0;
            M->lim[tid] = lim;
        }
        if (__syncthreads_or(local_bad)) {                 // block ids checked, slot rows and queries in
            if (tid == 0) report(P.status, TTKV_STATUS_BLOCK_RANGE);
            bad = true;
        }
        if (bad) {
            empty_partial(slot);
            __syncthreads();
            continue;
        }
        issue_cf(0);
        issue_kv(0);
        if (tid == RP_TID && T.rope_smem) issue_rp(0);
        pend_cf = true; pend_kv0 = true;
        if (T.rope_smem) pend_rp = true;
        float s_up;
        if (P.dec_image) {
            // the decoder's operand image (ttkv_decoder_image): one bulk copy into bhi || blo, which
            // the MMA thread waits for before the segment's first reconstruction
            if (tid == MMA_TID) {
                const uint32_t bytes = uint32_t(2 * T.natom * ATOM_BYTES);
                mbar_expect_tx(&M->mb_dec, bytes);
                bulk_g2s(bhi, P.dec_image + int64_t(di) * P.image_stride + int64_t(h) * bytes, bytes, &M->mb_dec);
                pend_dec = true;
            }
            s_up = P.dec_scales[int64_t(di) * P.H + h];
        } else {
            float mx = 0.f;
            {
                const float4* d4 = reinterpret_cast<const float4*>(dec - t) + lane;
                const int64_t rs4 = dstride / 4;
                #pragma unroll
                for (int i = 0; i < MAX_R1 / 16; ++i) {
                    const int rr = w + 16 * i;
                    if (rr < P.r1) {
                        const float4 v = d4[rr * rs4];
                        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                    }
                }
            }
            mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
            if (lane == 0) M->maxabs[w] = mx;
            __syncthreads();
            // decoder slice (again, from L2, while the tile's copies fly): power-of-two scale so
            // max|D| * 2^-e lies in [2^13, 2^14), then fp16 hi + lo
            mx = 0.f;
            #pragma unroll
            for (int i = 0; i < NTHR / 32; ++i) mx = fmaxf(mx, M->maxabs[i]);
            int e = 0;
            if (mx > 0.f) e = int((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 13;
            e = max(-100, min(100, e));
            const float s_down = __uint_as_float(uint32_t(127 - e) << 23);   // 2^-e
            s_up = __uint_as_float(uint32_t(127 + e) << 23);                 // 2^e
            #pragma unroll
            for (int jc = 0; jc < DEC_CHUNKS; ++jc) {
                const int cidx = wg + NWG * jc;
                if (cidx < nchunk) {
                    float dv[8];
                    #pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int rr = cidx * 8 + k;
                        dv[k] = rr < P.r1 ? dec[rr * dstride] : 0.f;
                    }
                    uint32_t hw[4], lw[4];
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t hh[2], ll[2];
                        #pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            const float v = dv[2 * i + k] * s_down;
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

        }

        // ---- first tile: its coefficient block, its A, its reconstruction (TMEM columns 0..127)
        wait_cf();
        float csp_next = convert_a(t_begin + t < t_end) * s_up;        // coefficient scale x 2^e of the tile
        fence_async_smem();
        tc_before();
        __syncthreads();
        tc_after();
        const uint32_t taddr = M->tmem_base;
        const uint32_t t_row = taddr + (uint32_t(32 * (w & 3)) << 16);    // this warp's TMEM lanes
        if (tid == MMA_TID && pend_dec) {
            if (!mbar_wait(&M->mb_dec, ph_dec)) timed_out = true;
            else { ph_dec ^= 1u; pend_dec = false; }
        }
        if (tid == MMA_TID) issue_recon(taddr);
        if (n_tiles > 1) {                                              // every conversion of tile 0 is done
            issue_cf(1);
            pend_cf = true;
        }

        float o[HPW], corr_prev[HPW], m_prev[HPW], lsum[HPW];
        #pragma unroll
        for (int i = 0; i < HPW; ++i) { o[i] = 0.f; corr_prev[i] = 0.f; m_prev[i] = -INFINITY; lsum[i] = 0.f; }
        bool r_pending = true, pv_pending = false;

        for (int it = 0; it < n_tiles; ++it) {
            const int t0 = t_begin + it * TM;
            const bool has_next = it + 1 < n_tiles;
            const int kb = kv_buf(it);
            const int tok = t0 + t;
            const bool valid = tok < t_end;
            const unsigned char* kvrow = kvb + (size_t(kb) * TM + t) * T.kvrow;
            const uint32_t kv_off = uint32_t(kvrow - base);
            // the next tile's K/V fields, into the other buffer (read by the tile before this one)
            if (T.nkv == 2 && has_next) { issue_kv(it + 1); mark_kv(it + 1); }
            // the slot rows of tile it + 2 over those of tile it, whose copies went out a barrier
            // ago; read after this tile's first barrier
            if (wg == NWG - 1 && it + 2 < n_tiles) fill_rows(it + 2, t);
            const uint32_t rcol = uint32_t(it & 1) * 128u;                 // this tile's reconstruction columns
            const float csp = csp_next;

            // ---- this token's RoPE row from global memory when it is not staged (used in the epilogue)
            uint4 cosw[2], sinw[2];
            if (!T.rope_smem) {
                const uint16_t* trow = reinterpret_cast<const uint16_t*>(P.table) +
                                       int64_t(min(valid ? tok : t_begin, int(P.table_rows - 1))) * 128;
                #pragma unroll
                for (int hp = 0; hp < 2; ++hp) {
                    cosw[hp] = __ldg(reinterpret_cast<const uint4*>(trow + 16 * wg + 8 * hp));
                    sinw[hp] = __ldg(reinterpret_cast<const uint4*>(trow + 64 + 16 * wg + 8 * hp));
                }
            }

            // ---- K residual: code windows of the bitmap bytes of lanes [16wg, 16wg+16) and
            // [64+16wg, 64+16wg+16) (bytes 2wg+hp and 8+2wg+hp); the fields are cut in the epilogue
            wait_kv(kb);
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

            // ---- PV of the previous tile: each warpgroup folds its query heads into o
            if (pv_pending) {
                if (!mbar_wait(&M->mb_pv, ph_pv)) timed_out = true;
                else { ph_pv ^= 1u; pv_pending = false; }
                tc_after();
                if (wg < G && !__any_sync(0xffffffffu, timed_out)) {
                    #pragma unroll
                    for (int i = 0; i < HPW; ++i) {
                        const int g = wg + NWG * i;
                        if (g < G) {
                            const float dh = tmem_ld1(t_row + PV_COL + uint32_t(g));
                            const float dl = tmem_ld1(t_row + PV_COL + uint32_t(G + g));
                            tmem_wait_ld();
                            o[i] = fmaf(o[i], corr_prev[i], dh + dl);
                        }
                    }
                }
            }

            // ---- V^T (MN-major): lanes [32wg, 32wg+32) of this token as exact small integers
            float vrs;
            {
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
                    // each group's rank from the word directly: the four groups do not wait on each other
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
                    const int ch = 4 * wg + gi;                         // lanes 8ch..8ch+7, one 16-byte chunk
                    const uint32_t off = uint32_t((t >> 3) * 2048 + (ch >> 3) * 1024 + (t & 7) * 128 +
                                                  (((ch & 7) ^ (t & 7)) << 4));
                    *reinterpret_cast<uint4*>(apv + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
                vrs = valid ? f16_at(vrow + voff + 16 + P.v_pb) : 0.f;
            }

            // ---- MMA 1 of this tile done: A is free for the next tile's coefficients
            if (r_pending) {
                if (!mbar_wait(&M->mb_r, ph_r)) timed_out = true;
                else { ph_r ^= 1u; r_pending = false; }
            }
            tc_after();
            if (has_next) {
                wait_cf();
                csp_next = convert_a(t0 + TM + t < t_end) * s_up;
            }

            // ---- epilogue: rebuild, patch, rotate, partial scores over this warpgroup's lanes
            if (T.rope_smem) {
                wait_rp();
                // row t of each box: 16-byte block c stored at block c ^ (t & 7)
                const unsigned char* rc = rpb + t * 128;
                #pragma unroll
                for (int hp = 0; hp < 2; ++hp) {
                    const int c = (2 * wg + hp) ^ (t & 7);
                    cosw[hp] = *reinterpret_cast<const uint4*>(rc + 16 * c);
                    sinw[hp] = *reinterpret_cast<const uint4*>(rc + RP_BOX + 16 * c);
                }
            }
            float sp[8];
            #pragma unroll
            for (int g = 0; g < 8; ++g) sp[g] = 0.f;
            if (!__any_sync(0xffffffffu, timed_out)) {
                // two accumulators per query head (the yl and the yh terms): chains half as long
                float2 s2[G], s2h[G];
                #pragma unroll
                for (int g = 0; g < G; ++g) { s2[g] = make_float2(0.f, 0.f); s2h[g] = s2[g]; }
                const float2 csp2 = make_float2(csp, csp), krs2 = make_float2(krs, krs);
                #pragma unroll
                for (int hp = 0; hp < 2; ++hp) {                        // 8 RoPE pairs at a time
                    const int j0 = 16 * wg + 8 * hp;
                    float al[8], ah[8];
                    tmem_ld8(t_row + rcol + uint32_t(j0), al);
                    tmem_ld8(t_row + rcol + uint32_t(64 + j0), ah);
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
                        const float2 kl = f2fma(make_float2(rl[2 * i], rl[2 * i + 1]), krs2,
                                                f2mul(make_float2(al[2 * i], al[2 * i + 1]), csp2));
                        const float2 kh = f2fma(make_float2(rh[2 * i], rh[2 * i + 1]), krs2,
                                                f2mul(make_float2(ah[2 * i], ah[2 * i + 1]), csp2));
                        const float2 yl = f2fma(make_float2(-kh.x, -kh.y), sz, f2mul(kl, cz));
                        const float2 yh = f2fma(kl, sz, f2mul(kh, cz));
                        #pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const float4 qq = qs4[g * 32 + (j0 >> 1) + i];
                            s2[g] = f2fma(make_float2(qq.x, qq.y), yl, s2[g]);
                            s2h[g] = f2fma(make_float2(qq.z, qq.w), yh, s2h[g]);
                        }
                    }
                }
                #pragma unroll
                for (int g = 0; g < G; ++g) sp[g] = (s2[g].x + s2h[g].x) + (s2[g].y + s2h[g].y);
                tmem_st8(t_row + RED_COL + uint32_t(8 * wg), sp);     // partial scores -> TMEM
                tmem_wait_st();
            }

            const bool cf_refill = it + 2 < n_tiles;
            fence_async_smem();                                          // V^T, next A for the MMAs
            tc_before();
            if (__syncthreads_or(timed_out)) { timed_out = true; break; }
            tc_after();

            // ---- MMA 1 of the next tile into the other reconstruction columns (under the softmax
            // and the next tile's decode), and the refills of the staging units this tile released
            if (has_next) {
                if (tid == MMA_TID) issue_recon(taddr + (rcol ^ 128u));
                r_pending = true;
            }
            if (T.nkv == 1 && has_next) { issue_kv(it + 1); mark_kv(it + 1); }   // the buffer is free now
            if (cf_refill) { issue_cf(it + 2); pend_cf = true; }
            if (T.rope_smem && has_next) {
                if (tid == RP_TID) issue_rp(it + 1);
                pend_rp = true;
            }

            // ---- online softmax over the tile: warpgroup wg owns query heads wg, wg + NWG, ... The tile
            // max is one warp reduction and one warpgroup barrier; each thread keeps the running sum
            // of its own tokens (rescaled with the max), reduced once after the last tile
            if (wg < G) {
                float sc[HPW], m_new[HPW], corr[HPW];
                #pragma unroll
                for (int i = 0; i < HPW; ++i) {
                    const int g = wg + NWG * i;
                    sc[i] = -INFINITY; m_new[i] = -INFINITY; corr[i] = 0.f;
                    if (g < G) {
                        float v = 0.f;
                        #pragma unroll
                        for (int c = 0; c < NWG; ++c) v += tmem_ld1(t_row + RED_COL + uint32_t(8 * c + g));
                        tmem_wait_ld();
                        sc[i] = (valid && tok < M->lim[g]) ? v * scale : -INFINITY;
                        const float mxg = warp_max(sc[i]);
                        if (lane == 0) M->red_max[w & 3][g] = mxg;
                    }
                }
                wg_sync(wg);
                #pragma unroll
                for (int i = 0; i < HPW; ++i) {
                    const int g = wg + NWG * i;
                    if (g < G) {
                        const float tmax = fmaxf(fmaxf(M->red_max[0][g], M->red_max[1][g]),
                                                 fmaxf(M->red_max[2][g], M->red_max[3][g]));
                        const float m_old = M->m[g];
                        m_new[i] = fmaxf(m_old, tmax);
                        const float pg = (m_new[i] == -INFINITY || sc[i] == -INFINITY) ? 0.f : expf(sc[i] - m_new[i]);
                        corr[i] = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new[i]);
                        lsum[i] = fmaf(lsum[i], corr[i], pg);
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
                }
                #pragma unroll
                for (int i = 0; i < HPW; ++i) { corr_prev[i] = corr[i]; m_prev[i] = m_new[i]; }
            }
            fence_async_smem();
            tc_before();
            __syncthreads();
            tc_after();
            // running max of each query head (every thread of its warpgroup has read the old one)
            if (wg < G && t == 0) {
                #pragma unroll
                for (int i = 0; i < HPW; ++i) {
                    const int g = wg + NWG * i;
                    if (g < G) M->m[g] = m_prev[i];
                }
            }

            // ---- MMA 2 of this tile: O^T = V^T . P', read back during the next tile
            if (tid == MMA_TID) issue_pv(taddr + PV_COL);
            pv_pending = true;
        }

        // ---- the last tile's PV
        if (!timed_out && pv_pending) {
            if (!mbar_wait(&M->mb_pv, ph_pv)) timed_out = true;
            else { ph_pv ^= 1u; pv_pending = false; }
            tc_after();
            if (wg < G && !__any_sync(0xffffffffu, timed_out)) {
                #pragma unroll
                for (int i = 0; i < HPW; ++i) {
                    const int g = wg + NWG * i;
                    if (g < G) {
                        const float dh = tmem_ld1(t_row + PV_COL + uint32_t(g));
                        const float dl = tmem_ld1(t_row + PV_COL + uint32_t(G + g));
                        tmem_wait_ld();
                        o[i] = fmaf(o[i], corr_prev[i], dh + dl);
                    }
                }
            }
        }
        // the softmax denominators: each owning warp's token sums, added up across its warpgroup
        if (wg < G) {
            #pragma unroll
            for (int i = 0; i < HPW; ++i) {
                const int g = wg + NWG * i;
                if (g < G) {
                    float sum = lsum[i];
                    #pragma unroll
                    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                    if (lane == 0) M->red_sum[w & 3][g] = sum;
                }
            }
        }
        // written before the set-up's barriers; read before this barrier, after which thread 0 may
        // start the next segment
        const int64_t slot_e = M->seg_slot;
        timed_out = __syncthreads_or(timed_out);

        r_pending_any = r_pending;
        pv_pending_any = pv_pending;
        // ---- this segment's partials: slot = virtual share + pair index (one per (share, pair))
        if (wg < G) {
            #pragma unroll
            for (int i = 0; i < HPW; ++i) {
                const int g = wg + NWG * i;
                if (g < G) P.part_o[(slot_e * G + g) * 128 + t] = timed_out ? 0.f : o[i];
            }
        }
        if (tid < G) {
            P.part_ml[(slot_e * G + tid) * 2 + 0] = timed_out ? -INFINITY : M->m[tid];
            const float l = M->red_sum[0][tid] + M->red_sum[1][tid] + M->red_sum[2][tid] + M->red_sum[3][tid];
            P.part_ml[(slot_e * G + tid) * 2 + 1] = timed_out ? 0.f : l;
        }
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
    }

    // ---- drain and release: anything still in flight gets one more bounded wait before TMEM and
    // the shared memory are released
    if (timed_out) {
        if (tid == 0) report(P.status, TTKV_STATUS_TIMEOUT);
        if (r_pending_any) mbar_wait(&M->mb_r, ph_r);
        if (pv_pending_any) mbar_wait(&M->mb_pv, ph_pv);
        if (pend_cf) mbar_wait(&M->mb_cf, par_cf);
        if (pend_rp) mbar_wait(&M->mb_rp, par_rp);
        if (pend_kv0) mbar_wait(&M->mb_kv[0], par_kv0);
        if (pend_kv1) mbar_wait(&M->mb_kv[1], par_kv1);
        if (pend_dec) mbar_wait(&M->mb_dec, ph_dec);
    }
    tc_before();
    __syncthreads();
    tc_after();
    if (w == 0) tmem_dealloc(M->tmem_base, TMEM_COLS);
}

// Combine the segments of one (request, KV head, query head): thread = lane. The segments of
// pair p are the virtual shares whose unit ranges meet p's units [U, U + tiles), written at
// slots c + p.
__global__ void __launch_bounds__(128) merge_sk_kernel(const ReadParams P) {
    __shared__ long long red[2][4];
    const int g = blockIdx.x, hl = blockIdx.y, r = blockIdx.z, lane = threadIdx.x;
    const int nh = P.n_heads;
    pdl_wait();                                                // the decode's partials are written
    long long before = 0, all = 0;
    for (int i = lane; i < P.n_reqs; i += 128) {
        const int v = req_tiles(P.seq_lens[i]);
        all += v;
        if (i < r) before += v;
    }
    #pragma unroll
    for (int off = 16; off; off >>= 1) {
        before += __shfl_xor_sync(0xffffffffu, before, off);
        all += __shfl_xor_sync(0xffffffffu, all, off);
    }
    if ((lane & 31) == 0) { red[0][lane >> 5] = before; red[1][lane >> 5] = all; }
    __syncthreads();
    before = red[0][0] + red[0][1] + red[0][2] + red[0][3];
    all = red[1][0] + red[1][1] + red[1][2] + red[1][3];
    const int nt = req_tiles(P.seq_lens[r]);
    float v = 0.f;
    const long long n = (long long)P.n_ctas * virtual_shares(all * nh, P.n_ctas, P.block_size);
    // seq_lens above the bound the workspace was sized for: the decode wrote nothing
    if (nt > 0 && n + (long long)P.n_reqs * nh <= P.n_part_slots) {
        const long long T = all * nh;
        const long long U = before * nh + (long long)hl * nt;
        const long long c0 = ((U + 1) * n - 1) / T, c1 = ((U + nt) * n - 1) / T;
        const long long p = (long long)r * nh + hl;
        // a CTA whose share is empty (fewer units than CTAs) wrote nothing; with at least as many
        // units as shares no share is empty, and the two 64-bit divisions per share are skipped
        const bool some_empty = T < n;
        auto empty = [&](long long c) { return c * T / n == (c + 1) * T / n; };
        // one pass, eight shares' loads in flight at a time, the running max rescaling the sums
        constexpr int NF = 8;
        float M = -INFINITY, acc = 0.f, den = 0.f;
        for (long long c = c0; c <= c1; c += NF) {
            float ms[NF], ls[NF], os[NF];
            #pragma unroll
            for (int k = 0; k < NF; ++k) {
                const long long cc = c + k;
                const bool ok = cc <= c1 && !(some_empty && empty(cc));
                const long long row = (min(cc, c1) + p) * P.G + g;
                ms[k] = ok ? P.part_ml[row * 2] : -INFINITY;
                ls[k] = ok ? P.part_ml[row * 2 + 1] : 0.f;
                os[k] = ok ? P.part_o[row * 128 + lane] : 0.f;
            }
            #pragma unroll
            for (int k = 0; k < NF; ++k) {
                if (ms[k] == -INFINITY) continue;
                const float Mn = fmaxf(M, ms[k]);
                const float a = expf(M - Mn), b = expf(ms[k] - Mn);   // a = 0 while M is -inf
                acc = fmaf(acc, a, b * os[k]);
                den = fmaf(den, a, b * ls[k]);
                M = Mn;
            }
        }
        v = den > 0.f ? acc / den : 0.f;
    }
    if (!P.v_req) {
        const int head_q = (P.head_lo + hl) * P.G + g;
        const int64_t at = int64_t(r) * P.out_stride + int64_t(head_q) * 128 + lane;
        store_elt(P.out, P.out_dtype, at, v);
        // the fused all-gather: the same row at the same offset of every other rank's output
        for (int p = 0; p < P.n_peers; ++p)
            if (p != P.peer_rank) store_elt(P.peer_out[p], P.out_dtype, at, v);
    } else if (g < P.v_nq[r]) {                                // row g = (query jq, head gh)
        const int f = P.v_f0[r] + g, jq = f / P.g_real, gh = f - jq * P.g_real;
        store_elt(P.out, P.out_dtype, int64_t(P.v_qrow[r] + jq) * P.out_stride +
                                      int64_t((P.head_lo + hl) * P.g_real + gh) * 128 + lane, v);
    }
    if (P.n_peers > 0) {
        // the CTA counts itself on the local ticket (a GPU-scope acquire-release add, ordered after
        // the CTA's row stores, which the barrier makes this thread's); the launch's last CTA, which
        // has acquired every other CTA's count and with it their stores, posts the launch's arrivals
        // to every rank's signal word with one system-scope release reduction per rank
        __syncthreads();
        if (lane == 0) {
            const unsigned long long n = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
            unsigned long long t;
            asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(t) : "l"(P.peer_ticket), "l"(1ull) : "memory");
            if (t + 1 == n) {                                  // the last: reset for the next launch
                for (int p = 0; p < P.n_peers; ++p)
                    asm volatile("red.release.sys.global.add.u64 [%0], %1;" :: "l"(P.peer_sig[p]), "l"(n) : "memory");
                asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" :: "l"(P.peer_ticket), "l"(0ull) : "memory");
            }
        }
    }
}

// The row blocks of a continuation launch (ttkv_prefill_cont_paged on the tensor-core decode):
// request r's chunk has q_len * G (query, query head) rows, query-major; block v = (request
// v / nqb, rows [b * rows, b * rows + rows) with b = v % nqb). Per block: the positions its last
// query sees (its row count for the schedule), its request, the request's first query row, its
// number of rows, the position of the request's first query and its first row; a block past
// the request's rows gets none. Refuses q_len > seq_len.
__global__ void cont_blocks_kernel(const int32_t* seq_lens, const int32_t* q_start, const int32_t* q_len,
                                   int n_reqs, int nqb, int G, int rows, int32_t* v_seq, int32_t* v_req,
                                   int32_t* v_qrow, int32_t* v_nq, int32_t* v_pos, int32_t* v_f0,
                                   int32_t* status) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n_reqs * nqb) return;
    const int r = v / nqb, f0 = (v - r * nqb) * rows;
    const int seq = seq_lens[r], ql = q_len[r];
    int n = 0;
    if (ql < 0 || ql > seq) {
        if (f0 == 0) report(status, TTKV_STATUS_QUERY);
    } else {
        n = max(0, min(rows, ql * G - f0));
    }
    const int p0 = seq - ql;
    v_seq[v] = n > 0 ? p0 + (f0 + n - 1) / G + 1 : 0;
    v_req[v] = r;
    v_qrow[v] = q_start[r];
    v_nq[v] = n;
    v_pos[v] = p0;
    v_f0[v] = f0;
}

// The decoders' operand images (ttkv_decoder_image): grid (decoders, KV heads), thread t = column
// t of the head's slice. The same scale and split as the decode's own staging, byte for byte, in
// the layout of its bhi || blo shared-memory region.
__global__ void __launch_bounds__(128) decoder_image_kernel(const float* dec, int64_t dec_stride, int r1, int H,
                                                            int kp16, int natom, unsigned char* image,
                                                            int64_t image_stride, float* scales) {
    __shared__ float wmax[4];
    const int n = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
    const float* col = dec + int64_t(n) * dec_stride + h * 128 + t;
    const int64_t rs = int64_t(H) * 128;
    float mx = 0.f;
    for (int rr = 0; rr < r1; ++rr) mx = fmaxf(mx, fabsf(col[rr * rs]));
    mx = warp_max(mx);
    if ((t & 31) == 0) wmax[t >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    int e = 0;
    if (mx > 0.f) e = int((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 13;
    e = max(-100, min(100, e));
    const float s_down = __uint_as_float(uint32_t(127 - e) << 23);
    unsigned char* bhi = image + int64_t(n) * image_stride + int64_t(h) * 2 * natom * ATOM_BYTES;
    unsigned char* blo = bhi + natom * ATOM_BYTES;
    for (int cidx = 0; cidx < kp16 / 8; ++cidx) {
        uint32_t hw[4], lw[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t hh[2], ll[2];
            #pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int rr = cidx * 8 + 2 * i + k;
                const float v = rr < r1 ? col[rr * rs] * s_down : 0.f;
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
    if (t == 0) scales[int64_t(n) * H + h] = __uint_as_float(uint32_t(127 + e) << 23);
}

// ------------------------------------------------------------------ host plan
// Bytes of one decoder's image: per KV head the hi and lo operand atoms.
inline size_t image_bytes(const ttkv_layout_t* lay) {
    const int kp16 = (lay->r1 + 15) / 16 * 16;
    return size_t(lay->H) * 2 * ((kp16 + 63) / 64) * ATOM_BYTES;
}
inline int round_up(int x, int a) { return (x + a - 1) / a * a; }

// The shared-memory plan of decode_tc_kernel for a layout, or smem == 0 if it does not fit.
// Preference: two K/V buffers with staged RoPE rows, then one K/V buffer, then RoPE rows read
// from global memory.
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
    // each bitmap is read as the two 16-byte blocks holding it
    T.kr = std::max(kr, 32);
    T.vr = std::max(vr, 32);
    // row pitches an odd number of 16-byte blocks: a warp's 32 rows then spread over all banks
    T.kvrow = T.kr + T.vr;
    if (((T.kvrow >> 4) & 1) == 0) T.kvrow += 16;
    // coefficient rows: an odd number of blocks as they are, a multiple of 8 XOR-swizzled, else padded
    const int cch = T.cb >> 4;
    T.cf_swz = (cch % 8 == 0) ? 7 : 0;
    T.cf_pitch = T.cb + ((cch & 1) == 0 && cch % 8 != 0 ? 16 : 0);
    const int atoms = T.natom * ATOM_BYTES;
    const int q_bytes = round_up(G * 128 * 4, 128);
    const int misc = round_up(int(sizeof(TcMisc)), 128);
    const int pref[4][2] = {{2, 1}, {1, 1}, {2, 0}, {1, 0}};      // {K/V buffers, staged RoPE}
    for (const auto& pr : pref) {
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
        T.off_cf = off; off += TM * T.cf_pitch;
        T.off_kv = off; off += pr[0] * TM * T.kvrow + KV_PAD;      // code windows read a few bytes past
        off = round_up(off, 1024);                                 // a 128-byte-swizzled TMA box
        T.off_rp = off; off += pr[1] * 2 * RP_BOX;
        T.nkv = pr[0];
        T.rope_smem = pr[1];
        T.smem = off + 1024;
        if (T.smem <= 227 * 1024) return T;
    }
    T.smem = 0;
    return T;
}

}  // namespace tc
