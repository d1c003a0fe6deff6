// tcgen05 / TMEM 3xTF32 GEMM with a fused elementwise epilogue (sm_100a).
//
// C[M,N] = epilogue(A[M,K] @ B[K,N], leaves...) in fp32 accuracy from
// TF32 tensor-core products (Ootomo & Yokota, "Recovering single precision
// accuracy from Tensor Cores while surpassing the FP32 theoretical peak
// performance", 2022): x = hi + lo with hi = x rounded to nearest TF32
// (x - hi is then exact in fp32, |x - hi| <= 2^-11 |x|) and lo = x - hi
// rounded to nearest TF32; C ~= Ahi*Bhi + Ahi*Blo + Alo*Bhi (the lo*lo term,
// ~2^-22 relative, is dropped).
//
// Launches:
//  1-2. pb_split_rows / pb_split_transpose: each operand, read in place with
//     its strides (inputs, slices and strided views of them, transposes),
//     -> hi, lo in K-major rows of K padded to 32: A [M,K] -> [M,Kp] and
//     B [K,N] -> [N,Kp]. An operand contiguous along K takes the row pass,
//     one contiguous along M or N (B as stored, a transposed A) the tile
//     transpose.
//  3. pb_gemm_tc:         one 128x256 output tile per CTA, 320 threads.
//     warp 8 lane 0 issues TMA loads (64B swizzle, BK = 16 fp32 = one 64-byte
//     swizzle row) into a 4-stage ring of {Ahi, Alo, Bhi, Blo} tiles (48 KB
//     per stage, 192 KB in all: three stages are in flight while the MMAs
//     read the fourth, about 1.8 us of tensor work, enough to cover TMA
//     latency from L2 or HBM); warp 9
//     allocates 512 TMEM columns and its lane 0 issues tcgen05.mma
//     (kind::tf32, M=128, N=256, K=8; 3 products x 2 k-steps per stage),
//     committing each stage back to the producer. With PB_PAIR (the
//     default wherever M has two or more 128-row tiles) a cluster of two
//     CTAs computes a 256x256 tile with cta_group::2 MMAs over 32-wide
//     k-blocks (see the PB_PAIR notes in the device source).
//     Accumulation: the tensor core's fp32 accumulator loses low-order bits
//     on every MMA it adds into, so one accumulator over all of K (1024
//     k-steps at K = 8192) drifts ~6e-5 relative -- five times an fp32 FMA
//     chain. Here the MMAs of each period of 4 k-blocks (64 of K) start from
//     zero in one of two 256-column TMEM buffers (p % 2), and eight warps
//     that are otherwise idle until the epilogue drain the finished period
//     with tcgen05.ld into per-thread fp32 sums (round to nearest) while the
//     MMAs fill the other buffer; the MMA thread reuses a buffer only after
//     its drain has arrived on that buffer's barrier. Warp w drains TMEM
//     lanes 32(w%4)..+31 (its tile rows) and column half w/4, then applies
//     the fused epilogue to its sums and stores.
// Every mbarrier wait is bounded (clock64 budget); on expiry the kernel
// records a code in the device error word, stops issuing, waits (bounded)
// for its own copies and MMAs in flight, frees its TMEM and returns.
// No TMA multicast is used anywhere.
#include "lower.hpp"

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <sstream>

namespace porch::detail {

    namespace {

        constexpr int kBM = 128;
        constexpr int kBN = 256;
        constexpr int kBK = 16;
        constexpr int kStages = 4;
        constexpr int kPairStages = 3;

        const char* gemm_device_source() {
            return R"PB(
#define PB_BM 128
#define PB_BN 256
// PB_PAIR: a cluster of two CTAs (on one SM pair) computes a 256 x 256
// tile with cta_group::2 MMAs: each CTA holds its own 128 rows of A and
// half (128 rows of N) of B, and its own 128 x 256 accumulator in TMEM.
// Its k-blocks are 32 fp32 wide (one 128-byte swizzle row; 8-row groups
// 1024 B apart) in 3 stages of 64 KB; one CTA per tile uses 16-wide
// k-blocks (64-byte swizzle, 512 B groups) in 4 stages of 48 KB.
#ifdef PB_PAIR
#define PB_CTAS 2
#define PB_BK 32
#define PB_STAGES 3
#define PB_SWIZZLE 2
#define PB_SBO 1024
#else
#define PB_CTAS 1
#define PB_BK 16
#define PB_STAGES 4
#define PB_SWIZZLE 4
#define PB_SBO 512
#endif
#define PB_BNH (PB_BN / PB_CTAS)
#define PB_TILE_A_BYTES (PB_BM * PB_BK * 4)
#define PB_TILE_B_BYTES (PB_BNH * PB_BK * 4)
#define PB_STAGE_BYTES (2 * PB_TILE_A_BYTES + 2 * PB_TILE_B_BYTES)
#define PB_WAIT_CYCLES 4000000000ll

struct __align__(64) pb_tmap { unsigned long long opaque[16]; };

static __device__ __forceinline__ pb_u32 pb_smem(const void* p) {
    return (pb_u32)__cvta_generic_to_shared(p);
}

static __device__ __forceinline__ void pb_mbar_init(pb_u32 bar, pb_u32 count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}

static __device__ __forceinline__ void pb_mbar_arrive(pb_u32 bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}

static __device__ __forceinline__ void pb_mbar_expect_tx(pb_u32 bar, pb_u32 bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}

// Rank of this CTA in its cluster (0 without PB_PAIR) and the
// shared::cluster address of the same shared variable in CTA `rank`.
static __device__ __forceinline__ pb_u32 pb_cta_rank() {
#ifdef PB_PAIR
    pb_u32 r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
#else
    return 0u;
#endif
}

static __device__ __forceinline__ pb_u32 pb_mapa(pb_u32 addr, pb_u32 rank) {
    pb_u32 r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// All threads of both CTAs of the pair (release / acquire; the forms that
// do not need the warp converged).
static __device__ __forceinline__ void pb_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}

// Arrivals on an mbarrier of either CTA of the pair (shared::cluster address).
static __device__ __forceinline__ void pb_mbar_arrive_cl(pb_u32 bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(bar) : "memory");
}

// Counts `bytes` as landed on a local barrier (for bytes that will never come).
static __device__ __forceinline__ void pb_mbar_complete_tx(pb_u32 bar, pb_u32 bytes) {
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}

static __device__ __forceinline__ pb_u32 pb_mbar_try(pb_u32 bar, pb_u32 parity) {
    pb_u32 ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok;
}

// Bounded wait: false when the budget ran out or another role (of this
// CTA or, in a pair, of the other CTA) aborted.
static __device__ __forceinline__ bool pb_wait_for(pb_u32 bar, pb_u32 parity, volatile int* abort_flag,
                                                   int* err, int site, long long budget) {
    const long long start = clock64();
    for (;;) {
        if (pb_mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - start > budget) {
            *abort_flag = 1;
#ifdef PB_PAIR
            {   // the other CTA of the pair stops too (its flag, through distributed shared memory)
                pb_u64 peer;
                asm volatile("mapa.u64 %0, %1, %2;" : "=l"(peer) : "l"((pb_u64)abort_flag), "r"(pb_cta_rank() ^ 1u));
                *(volatile int*)peer = 1;
            }
#endif
            if (atomicCAS(err, 0, 0x7c00 + site) == 0) {
                err[1] = site;
                err[2] = (int)blockIdx.x;
            }
            return false;
        }
    }
}

static __device__ __forceinline__ bool pb_wait(pb_u32 bar, pb_u32 parity, volatile int* abort_flag, int* err,
                                               int site) {
    return pb_wait_for(bar, parity, abort_flag, err, site, PB_WAIT_CYCLES);
}

// Teardown wait: bounded, records nothing.
static __device__ __forceinline__ void pb_wait_quiet(pb_u32 bar, pb_u32 parity) {
    const long long start = clock64();
    while (!pb_mbar_try(bar, parity) && clock64() - start <= PB_WAIT_CYCLES) {
    }
}

// An int in the other CTA of the pair (distributed shared memory).
static __device__ __forceinline__ int pb_peer_int(const int* p) {
    pb_u64 q;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(q) : "l"((pb_u64)p), "r"(pb_cta_rank() ^ 1u));
    return *(const volatile int*)q;
}

// Tile load into this CTA's shared memory; completion is counted on `bar`,
// which in a pair is the first CTA's barrier (a shared::cluster address).
static __device__ __forceinline__ void pb_tma_load(pb_u32 dst, const pb_tmap* map, pb_u32 bar, int x, int y) {
#ifdef PB_PAIR
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(dst), "l"((unsigned long long)map), "r"(bar), "r"(x), "r"(y) : "memory");
#else
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(dst), "l"((unsigned long long)map), "r"(bar), "r"(x), "r"(y) : "memory");
#endif
}

// tcgen05 shared-memory matrix descriptor: K-major, one swizzle row per
// tile row (64 bytes = 16 fp32 of K, or 128 bytes = 32 with PB_PAIR), 8-row
// groups PB_SBO bytes apart, start address in 16-byte units (a k-step of 8
// fp32 advances it by 32 bytes within the swizzle row). Tiles start on
// 1024-byte boundaries, so the swizzle phase (base offset field) is 0.
static __device__ __forceinline__ pb_u64 pb_desc(pb_u32 addr) {
    pb_u64 d = 0;
    d |= (pb_u64)((addr & 0x3FFFFu) >> 4);
    d |= (pb_u64)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (pb_u64)(PB_SBO >> 4) << 32; // stride byte offset
    d |= (pb_u64)1 << 46;             // fixed 0b001
    d |= (pb_u64)PB_SWIZZLE << 61;    // 64- or 128-byte swizzle
    return d;
}

// Instruction descriptor: D f32, A/B tf32, both K-major, N>>3, M>>4 (M of
// the whole MMA: 256 for a pair).
#define PB_IDESC ((1u << 4) | (2u << 7) | (2u << 10) | ((pb_u32)(PB_BN >> 3) << 17) | ((pb_u32)((PB_BM * PB_CTAS) >> 4) << 24))

// Issued by one thread (of the first CTA in a pair); the descriptors name
// this CTA's shared memory, and a pair's MMA reads the other CTA's A and B
// halves at the same offsets.
static __device__ __forceinline__ void pb_mma(pb_u32 tmem, pb_u64 a, pb_u64 b, pb_u32 accumulate) {
#ifdef PB_PAIR
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
                 :: "r"(tmem), "l"(a), "l"(b), "r"(PB_IDESC), "r"(accumulate) : "memory");
#else
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
                 :: "r"(tmem), "l"(a), "l"(b), "r"(PB_IDESC), "r"(accumulate) : "memory");
#endif
}

// Arrives on `bar` (a local shared address) once the MMAs issued so far have
// completed: in a pair, on that barrier in both CTAs.
static __device__ __forceinline__ void pb_commit(pb_u32 bar) {
#ifdef PB_PAIR
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(pb_mapa(bar, 0u)) : "memory");
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(pb_mapa(bar, 1u)) : "memory");
#else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
#endif
}

// The same, on this CTA's barrier only.
static __device__ __forceinline__ void pb_commit_local(pb_u32 bar) {
#ifdef PB_PAIR
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(pb_mapa(bar, pb_cta_rank())) : "memory");
#else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
#endif
}

static __device__ __forceinline__ float pb_tf32_rn(float x) {
    pb_u32 r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// hi = x rounded to TF32 (truncated instead where rounding would overflow);
// x - hi is then exact in fp32 and |x - hi| <= 2^-11 |x|.
static __device__ __forceinline__ float pb_tf32_hi(float x) {
    const float r = pb_tf32_rn(x);
    return isinf(r) && !isinf(x) ? __uint_as_float(__float_as_uint(x) & 0xFFFFE000u) : r;
}

// Named barrier 1 over the 256 drain/epilogue threads (warps 0-7), with and
// without an AND of a predicate.
static __device__ __forceinline__ void pb_bar_drain() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
static __device__ __forceinline__ bool pb_bar_all(bool v) {
    pb_u32 r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 1, 256, q;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(r) : "r"((pb_u32)v) : "memory");
    return r != 0;
}

#define PB_TMEM_LD32(taddr, v)                                                                   \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15," \
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"       \
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), \
                   "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), \
                   "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), \
                   "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), \
                   "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])                              \
                 : "r"(taddr))
)PB";
        }

        std::string hex8(const std::string& s) {
            uint64_t h = 0xcbf29ce484222325ULL;
            for (unsigned char c : s) {
                h ^= c;
                h *= 0x100000001b3ULL;
            }
            char b[20];
            std::snprintf(b, sizeof b, "%08x", static_cast<unsigned>(h >> 32));
            return b;
        }

        std::atomic<bool> g_test_stall{false};

        bool tensor_cores_disabled() {
            const char* v = std::getenv("PORCH_B200_GEMM");
            return v != nullptr && std::string{v} == "simt";
        }

        bool gemm_pairs_enabled() {
            const char* v = std::getenv("PORCH_B200_GEMM");
            return v == nullptr || std::string{v} != "single";
        }

    } // namespace

    bool tensor_core_gemm(int64_t M, int64_t N, int64_t K) {
        return !tensor_cores_disabled() && M >= 1 && N >= 1 && K >= 1 && M * N * K >= (int64_t{1} << 27) &&
               M <= (int64_t{1} << 30) && N <= (int64_t{1} << 30) && K <= (int64_t{1} << 30);
    }

    std::string gemm_form_key() {
        const char* v = std::getenv("PORCH_B200_GEMM");
        return v == nullptr ? std::string{} : "|gemm=" + std::string{v};
    }

    void set_test_gemm_stall(bool on) { g_test_stall.store(on); }
    bool test_gemm_stall() { return g_test_stall.load(); }

    int lowerer::emit_gemm_tc(int id, const box& b, kernel& k, const gemm_operand& A,
                              const gemm_operand& B, int64_t M, int64_t N, int64_t K, int* nonfinite,
                              int* row_partials, int out_temp, int64_t out_off, gemm_temps* shared,
                              const split_output* so, const gemm_batches* batches) {
        const bool softmax = row_partials != nullptr;
        if (so != nullptr && (softmax || N % 32 != 0 || so->kp != N)) return -1;
        (void)id;
        // Grouped batches (plain or fused elementwise epilogues only): the
        // tensor cores pay off on the total work, and the stacked operand
        // rows (nb * M, nb * N) must stay within a tensor map's range.
        const int64_t nb = batches != nullptr ? batches->count : 1;
        if (nb > 1 && (softmax || so != nullptr || out_off != 0 || N == 1 || nb * M > (int64_t{1} << 30) ||
                       nb * N > (int64_t{1} << 30) || !tensor_core_gemm(nb * M, N, K)))
            return -1;
        if (nb == 1 && !tensor_core_gemm(M, N, K)) return -1;
        // Any M, N, K. The K-major hi/lo arrays have padded rows (16-byte
        // TMA strides whatever K is); edge tiles read zeros past M, N and K
        // (TMA out-of-bounds fill) and mask their stores; when N is not a
        // multiple of 4 the epilogue loads and stores one float at a time.
        if (M < 1 || N < 1 || K < 1) return -1;
        if (nb * M * N * K < (int64_t{1} << 27)) return -1;
        if (M > (int64_t{1} << 30) || N > (int64_t{1} << 30) || K > (int64_t{1} << 30)) return -1;
        rank_ = 2;

        // The K-major hi/lo arrays have rows of Kp = K rounded up to 32
        // (zeros past K), so every row starts on a 128-byte line and the
        // TMA boxes (64-byte rows) never straddle one.
        const int64_t Kp = (K + 31) / 32 * 32;
        gemm_temps own;
        gemm_temps& tt = shared != nullptr ? *shared : own;
        auto need = [&](int& t, size_t bytes) {
            if (t < 0) t = new_temp(bytes);
        };
        need(tt.a_hi, static_cast<size_t>(nb * M * Kp) * 4);
        need(tt.a_lo, static_cast<size_t>(nb * M * Kp) * 4);
        need(tt.b_hi, static_cast<size_t>(nb * N * Kp) * 4);
        need(tt.b_lo, static_cast<size_t>(nb * N * Kp) * 4);
        need(tt.nf, 256);
        need(tt.fa, 256);
        need(tt.fb, 256);
        const int a_hi = tt.a_hi, a_lo = tt.a_lo, b_hi = tt.b_hi, b_lo = tt.b_lo;
        const int out = so != nullptr ? so->hi : out_temp >= 0 ? out_temp : new_temp(static_cast<size_t>(M * N) * 4);
        // Set by the split kernels when an operand holds Inf or NaN; the
        // tensor-core kernels then leave the output to the CUDA-core GEMM
        // that follows them in the plan.
        // Each split flags its own operand (fa, fb: a kept split keeps its
        // flag); a one-thread merge then sets nf = fa | fb.
        const int nf = tt.nf, fa = tt.fa, fb = tt.fb;
        *nonfinite = nf;
        auto temp_arg = [](int t) {
            kernel_arg a;
            a.kind = arg_kind::temp;
            a.index = t;
            return a;
        };
        {
            launch_spec l;
            l.name = "pb_nonfinite_clear";
            l.source = std::string(kernel_prelude()) +
                       "extern \"C\" __global__ void pb_nonfinite_clear(int* fa, int* fb) { fa[0] = 0; fb[0] = 0; }\n";
            l.schedule = "clear the operands' non-finite flags";
            l.grid = {1, 1, 1};
            l.block = {1, 1, 1};
            kernel_arg ca, cb;
            ca.kind = cb.kind = arg_kind::flag_clear;
            ca.index = tt.a_ready ? nf : fa; // a flag set by A's producer is not cleared
            cb.index = fb;
            ca.value = cb.value = static_cast<uint64_t>(nf); // harmless stand-in for a kept flag
            l.args = {ca, cb};
            finish_kernel(l);
            p_.launches.push_back(std::move(l));
        }

        // ---- 1-2. split A and B into K-major hi/lo ---------------------------
        // Each operand is read in place as a K-major source: rows r (A: its
        // M rows; B: its N columns), element (r, k) at off + r * sr + k * sk.
        // Contiguous along k: a row pass (float4 when rows start 16-byte
        // aligned); contiguous along r (a transposed operand, or B as
        // stored): 64 x 64 tiles through shared memory so both the loads
        // and the K-major stores stay coalesced; otherwise the same tiles
        // with strided loads.
        // zb > 1: zb operands zx elements apart (blockIdx.z), their halves
        // stacked R rows apart (the transposing split of batched B).
        auto emit_split = [&](const std::string& what, const gemm_operand& X, int64_t R, int64_t sr, int64_t sk,
                              int hi_t, int lo_t, int flag_t, int64_t zb = 1, int64_t zx = 0) {
            std::ostringstream src;
            src << kernel_prelude() << gemm_device_source();
            launch_spec l;
            if (sk == 1) {
                const int64_t n4 = R * Kp / 4;
                src << "extern \"C\" __global__ void __launch_bounds__(256) pb_split_rows(const float* __restrict__ x, "
                       "float* __restrict__ hi, float* __restrict__ lo, int* __restrict__ nf) {\n"
                    << "    for (pb_u64 i = (pb_u64)blockIdx.x * 256u + threadIdx.x; i < " << n4
                    << "ull; i += (pb_u64)gridDim.x * 256u) {\n";
                if (Kp == K && sr == K && X.off == 0) {
                    src << "        const float4 v = pb_ld4(x + 4 * i);\n";
                } else if (K % 4 == 0 && sr % 4 == 0 && X.off % 4 == 0) {
                    src << "        const pb_u64 r = i / " << Kp / 4 << "ull, c = i % " << Kp / 4 << "ull;\n"
                        << "        const float4 v = c < " << K / 4 << "ull ? pb_ld4(x + " << X.off << "ull + r * " << sr
                        << "ull + 4 * c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);\n";
                } else {
                    // Rows not 16-byte aligned: one float at a time.
                    src << "        const pb_u64 r = i / " << Kp / 4 << "ull, c = 4 * (i % " << Kp / 4 << "ull);\n"
                        << "        const float* xr = x + " << X.off << "ull + r * " << sr << "ull;\n"
                        << "        float4 v;\n"
                        << "        v.x = c < " << K << "ull ? pb_ld(xr + c) : 0.0f;\n"
                        << "        v.y = c + 1 < " << K << "ull ? pb_ld(xr + c + 1) : 0.0f;\n"
                        << "        v.z = c + 2 < " << K << "ull ? pb_ld(xr + c + 2) : 0.0f;\n"
                        << "        v.w = c + 3 < " << K << "ull ? pb_ld(xr + c + 3) : 0.0f;\n";
                }
                src << "        if (!(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w))) atomicOr(nf, 1);\n"
                    << "        float4 h, l;\n"
                    << "        h.x = pb_tf32_hi(v.x); l.x = pb_tf32_rn(v.x - h.x);\n"
                    << "        h.y = pb_tf32_hi(v.y); l.y = pb_tf32_rn(v.y - h.y);\n"
                    << "        h.z = pb_tf32_hi(v.z); l.z = pb_tf32_rn(v.z - h.z);\n"
                    << "        h.w = pb_tf32_hi(v.w); l.w = pb_tf32_rn(v.w - h.w);\n"
                    << "        pb_st4(hi + 4 * i, h);\n        pb_st4(lo + 4 * i, l);\n    }\n}\n";
                l.name = "pb_split_rows";
                l.schedule = "3xTF32 split of " + what + " (hi = rn(x), lo = rn(x - hi))";
                l.grid = {static_cast<uint32_t>(std::min<int64_t>((n4 + 255) / 256, 148 * 16)), 1, 1};
            } else {
                // Tile (k0.., r0..): loads walk r (coalesced when sr == 1),
                // stores walk k of the K-major output.
                src << "extern \"C\" __global__ void __launch_bounds__(256) pb_split_transpose(const float* __restrict__ x, "
                       "float* __restrict__ hi, float* __restrict__ lo, int* __restrict__ nf) {\n"
                    << (zb > 1 ? "    x += (pb_u64)blockIdx.z * " + std::to_string(zx) + "ull;\n    hi += (pb_u64)blockIdx.z * " +
                                     std::to_string(R * Kp) + "ull;\n    lo += (pb_u64)blockIdx.z * " +
                                     std::to_string(R * Kp) + "ull;\n"
                               : std::string{})
                    << "    __shared__ float t[64][65];\n"
                    << "    const pb_u64 k0 = (pb_u64)blockIdx.y * 64u, n0 = (pb_u64)blockIdx.x * 64u;\n"
                    << "    #pragma unroll\n    for (int u = 0; u < 16; ++u) {\n"
                    << "        const pb_u32 r = threadIdx.x / 64u + 4u * u, c = threadIdx.x % 64u;\n"
                    << "        t[r][c] = (k0 + r < " << K << "ull && n0 + c < " << R << "ull) ? pb_ld(x + " << X.off
                    << "ull + (k0 + r) * " << sk << "ull + (n0 + c)" << (sr == 1 ? std::string{} : " * " + std::to_string(sr) + "ull")
                    << ") : 0.0f;\n    }\n"
                    << "    __syncthreads();\n"
                    << "    #pragma unroll\n    for (int u = 0; u < 16; ++u) {\n"
                    << "        const pb_u32 r = threadIdx.x / 64u + 4u * u, c = threadIdx.x % 64u;\n"
                    << "        if (n0 + r >= " << R << "ull || k0 + c >= " << Kp << "ull) continue;\n"
                    << "        const float v = t[c][r];\n"
                    << "        if (!isfinite(v)) atomicOr(nf, 1);\n"
                    << "        const float h = pb_tf32_hi(v);\n"
                    << "        const pb_u64 o = (n0 + r) * " << Kp << "ull + k0 + c;\n"
                    << "        hi[o] = h;\n        lo[o] = pb_tf32_rn(v - h);\n    }\n}\n";
                l.name = "pb_split_transpose";
                l.schedule = "3xTF32 split of " + what + " with transpose to K-major";
                l.grid = {static_cast<uint32_t>((R + 63) / 64), static_cast<uint32_t>((Kp + 63) / 64),
                          static_cast<uint32_t>(zb)};
            }
            l.source = src.str();
            l.args = {X.arg, temp_arg(hi_t), temp_arg(lo_t), temp_arg(flag_t)};
            if (X.arg.kind == arg_kind::slot) {
                // A realised input: its storage may keep this split.
                l.cache_slot = X.arg.index;
                l.cache_key = "split R" + std::to_string(R) + " K" + std::to_string(K) + " Kp" + std::to_string(Kp) +
                              " off" + std::to_string(X.off + X.arg.elem_offset) + " sr" + std::to_string(sr) +
                              " sk" + std::to_string(sk) +
                              (zb > 1 ? " z" + std::to_string(zb) + "x" + std::to_string(zx) : std::string{});
                l.cache_temps = {hi_t, lo_t, flag_t};
            }
            finish_kernel(l);
            p_.launches.push_back(std::move(l));
        };
        // Batched operands are contiguous: A's rows of every batch form one
        // [nb * M, K] matrix; B's batches are transposed one per blockIdx.z.
        if (!tt.a_ready) emit_split("A", A, nb * M, A.s0, A.s1, a_hi, a_lo, fa);
        emit_split("B", B, N, B.s1, B.s0, b_hi, b_lo, fb, nb, K * N);
        {
            launch_spec l;
            l.name = "pb_nonfinite_merge";
            l.source = std::string(kernel_prelude()) +
                       "extern \"C\" __global__ void pb_nonfinite_merge(int* nf, const int* fa, const int* fb) "
                       "{ nf[0] = fa[0] | fb[0]; }\n";
            l.schedule = "merge the operands' non-finite flags";
            l.grid = {1, 1, 1};
            l.block = {1, 1, 1};
            l.args = {temp_arg(nf), temp_arg(fa), temp_arg(fb)};
            finish_kernel(l);
            p_.launches.push_back(std::move(l));
        }
        // ---- 3. tcgen05 GEMM + epilogue -------------------------------------
        std::vector<int> order;
        const std::string efn = emit_expr_function(b, "0", order);
        // CTA pairs (cta_group::2, 256 x 256 tiles) wherever there are at
        // least two 128-row tiles and pairing leaves no more than a sliver
        // of a pair idle; one CTA per 128 x 256 tile otherwise (or with
        // PORCH_B200_GEMM=single). Each CTA of a pair loads half of B for
        // the same MMAs (a third fewer bytes from L2 and through the tensor
        // core's shared-memory reads), with 32-wide k-blocks in a 128-byte
        // swizzle (3 stages of 64 KB): half the barrier round trips between
        // the two SMs per MMA. Measured on config 5 at the same clock:
        // 244-245 TFLOP/s against 222-223 for one CTA per tile. (With the
        // one-CTA form's 16-wide k-blocks in 6 stages the pair ran at
        // 216-220: the per-stage handshakes between the SMs left the tensor
        // pipe idle.) The results are bit-identical either way, except
        // under split-K when a part holds an odd number of 16-wide k-blocks
        // (a pair's parts are whole 32-wide k-blocks, so its split points
        // move by 16 of K).
        const int64_t tiles_m1 = (M + kBM - 1) / kBM;
        const bool pair = gemm_pairs_enabled() && tiles_m1 >= 2 && (tiles_m1 % 2 == 0 || tiles_m1 >= 8);
        const int ctas = pair ? 2 : 1;
        const int64_t slots = 148 / ctas; // work units resident at once
        const int64_t tiles_m = (M + kBM * ctas - 1) / (kBM * ctas), tiles_n = (N + kBN - 1) / kBN;
        const int64_t raw_kb = (K + kBK - 1) / kBK;
        const int group_m = 16 / ctas; // 16 rows of 128
        // Accumulation period in k-blocks. The drift of a tensor-core
        // accumulator grows with the number of MMAs added into one period
        // (6 per k-block: 3 products x 2 k-steps), independent of K, while
        // an fp32 FMA chain's error grows as sqrt(K); a period of at most
        // sqrt(K) / 2 k-blocks keeps ours about half the chain's at every K
        // (measured: one accumulator over 8192 of K drifts 5x the chain, a
        // period over all of K = 512 almost 5x). Capped at 32 (draining
        // costs a few percent per launch at 8), a power of two, at least 4.
        // A tile's last period may be shorter (it then drifts less).
        int period = 4;
        while (period < 32 && static_cast<double>(period * 2) <= std::sqrt(static_cast<double>(K)) / 2.0)
            period *= 2;
        // Split-K when the tiles leave most SMs idle (fewer tiles than half
        // of 148 SMs: a short batch, a thin row block): S K-ranges per tile
        // (a power of two up to 16, each at least 256 of K; the k-blocks
        // are padded to a multiple of S, past K the TMA loads read zeros,
        // which add exactly nothing), S chosen to fill whole waves best. Each unit
        // writes its raw partial tile; a second kernel sums the S partials
        // in split order and applies the fused epilogue. Measured on one
        // box: 16 tiles (128 x 4096 x 4096) 2.9x faster with S = 8; at 128
        // and 256 tiles splitting lost to the extra partial traffic, since
        // a part-filled last wave runs at a higher clock.
        const int64_t tiles = tiles_m * tiles_n;
        int64_t split = 1;
        auto wave_fill = [slots](int64_t u) {
            return static_cast<double>(u) / static_cast<double>(slots * ((u + slots - 1) / slots));
        };
        // The softmax epilogue can hand a split-K combine the whole row
        // softmax when a row fits one CTA's registers (16 float4 a thread).
        const bool softmax_split_ok = softmax && N % 1024 == 0 && N <= 16384;
        // One policy for both epilogues, so a softmax over a product and the
        // product realised alone sum K in the same parts.
        if (nb == 1 && tiles < slots / 2 && (!softmax || softmax_split_ok) && so == nullptr) {
            double best = static_cast<double>(tiles) / static_cast<double>(slots);
            for (int64_t s = 2; s <= 16; s *= 2) {
                if (raw_kb / s < 16) break;
                const int64_t u = tiles * s;
                const double eff = wave_fill(u);
                if (eff > best + 1e-9) {
                    best = eff;
                    split = s;
                }
            }
        } else if (nb == 1 && so == nullptr && (!softmax || softmax_split_ok) && tiles < 4 * slots && K > 4096) {
            // A few waves of long tiles whose last wave leaves SMs idle
            // (config 5's second GEMM per rank at 4 and 8 GPUs: 512 and 256
            // tiles, 86.5 % filled): split K in 2 or 4 when that fills the
            // waves clearly better and each part keeps >= 2048 of K (the
            // partials' extra traffic, 2 x S x M x N x 4 bytes, is then a
            // few percent of the tile's tensor time).
            double best = wave_fill(tiles);
            int64_t pick = 1;
            for (int64_t s = 2; s <= 4; s *= 2) {
                if (raw_kb / s < 128) break;
                const double eff = wave_fill(tiles * s);
                if (eff > best + 0.05) {
                    best = eff;
                    pick = s;
                }
            }
            split = pick;
        }
        const bool softmax_split = softmax && split > 1;
        int64_t kb_unit = (raw_kb + split - 1) / split;
        // A pair's k-blocks are 32 wide: whole ones per unit (past K the
        // loads read zeros). The periods keep the same length in K.
        if (pair) kb_unit = (kb_unit + 1) / 2 * 2;
        const int64_t units = tiles * split * nb;  // grouped batches: every batch's tiles
        const int part = split > 1 ? new_temp(static_cast<size_t>(split * M * ((N + 3) / 4 * 4)) * 4) : -1;
        // With split-K the combine does the whole softmax: no row partials.
        const int stats = softmax && !softmax_split ? new_temp(static_cast<size_t>(M * tiles_n) * 8) : -1;
        if (softmax) *row_partials = stats;
        std::ostringstream src;
        src << kernel_prelude() << (test_gemm_stall() ? "#define PB_TEST_STALL 1\n" : "")
            << (pair ? "#define PB_PAIR 1\n" : "") << "#define PB_PERIOD "
            << (pair ? period / 2 : period) << "\n#define PB_SPLIT " << split << "\n"
            << gemm_device_source() << efn;
        // Tile t -> output origin, tiles ordered in groups of group_m M-tiles
        // that sweep N (consecutive tiles, run at the same time by the
        // persistent CTAs, share A and B panels in L2).
        // With grouped batches, tile t of batch bt is unit bt * tiles + t.
        src << "static __device__ __forceinline__ void pb_tile_origin(pb_u32 t, int& m0, int& n0, pb_u32& bt) {\n"
            << (nb > 1 ? "    bt = t / " + std::to_string(tiles) + "u;\n    t -= bt * " + std::to_string(tiles) + "u;\n"
                       : std::string("    bt = 0u;\n"))
            << "    const pb_u32 tiles_m = " << tiles_m << "u, tiles_n = " << tiles_n << "u;\n"
            << "    const pb_u32 per_group = " << group_m << "u * tiles_n;\n"
            << "    const pb_u32 g = t / per_group, first_m = g * " << group_m << "u;\n"
            << "    const pb_u32 gm = (tiles_m - first_m) < " << group_m << "u ? (tiles_m - first_m) : " << group_m << "u;\n"
            << "    m0 = (int)((first_m + (t % per_group) % gm) * (PB_BM * PB_CTAS));\n"
            << "    n0 = (int)(((t % per_group) / gm) * PB_BN);\n"
            << "}\n";
        // Grouped batches: each tile's epilogue sees its batch's output and
        // leaves (the kernel's parameters carry a _g suffix).
        std::string batch_ptrs;
        if (nb > 1) {
            batch_ptrs = "            float* const out = out_g + (pb_u64)bt * " + std::to_string(M * N) + "ull;\n";
            for (size_t i = 0; i < k.leaves.size(); ++i) {
                const int64_t bs = i < batches->leaf_stride.size() ? batches->leaf_stride[i] : 0;
                batch_ptrs += "            const float* const in" + std::to_string(i) + " = in" + std::to_string(i) +
                              "_g" + (bs > 0 ? " + (pb_u64)bt * " + std::to_string(bs) + "ull" : std::string{}) +
                              ";\n";
            }
        }
        std::ostringstream body;
        // Persistent CTAs (one per SM) loop over tiles t = blockIdx.x,
        // + gridDim.x, ...; the k-block counter g and the period counter run
        // on across tiles, so the producer fetches the next tile's stages
        // and the MMAs start its first period while the eight drain warps
        // still run the previous tile's epilogue from their registers.
        // Roles (320 threads): warps 0-7 drain the accumulator periods and
        // run the epilogue (warp w: TMEM lane quadrant w % 4 = tile rows
        // 32(w%4).., column half w / 4), warp 8 lane 0 issues TMA, warp 9
        // allocates TMEM and its lane 0 issues the MMAs.
        body << "    if (*(const volatile int*)nf != 0) return;  // non-finite operand: CUDA-core GEMM\n"
             << "    extern __shared__ float4 pb_dyn_smem[];\n"
             << "    __shared__ __align__(8) unsigned long long full_bar[PB_STAGES], empty_bar[PB_STAGES];\n"
             << "    __shared__ __align__(8) unsigned long long accf[2], acce[2], done_bar;\n"
             << "    __shared__ pb_u32 tmem_slot;\n"
             << "    __shared__ int abort_flag;\n"
             << "    __shared__ int issued, consumed;\n"
             << "#ifdef PB_TEST_STALL\n    __shared__ __align__(8) unsigned long long stall_bar;\n#endif\n"
             << (softmax && !softmax_split ? "    __shared__ float sm_max[2][PB_BM], sm_sum[2][PB_BM];\n" : "")
             << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n"
             << "    const pb_u32 rank = pb_cta_rank();  // 1: the second CTA of a pair\n"
             << "    const pb_u32 base = (pb_smem(pb_dyn_smem) + 1023u) & ~1023u;\n"
             << "    const pb_u32 tiles = " << units << "u;  // work units: tiles x K splits\n"
             << "    if (threadIdx.x == 0) {\n"
             << "        abort_flag = 0;\n"
             << "        issued = 0;\n"
             << "        consumed = 0;\n"
             // In a pair the first CTA's full barriers count both CTAs'
             // bytes (the first CTA arms them for both), its acce barriers
             // both CTAs' drains.
             << "        for (int s = 0; s < PB_STAGES; ++s) { pb_mbar_init(pb_smem(&full_bar[s]), 1); pb_mbar_init(pb_smem(&empty_bar[s]), 1); }\n"
             << "        for (int b = 0; b < 2; ++b) { pb_mbar_init(pb_smem(&accf[b]), 1); pb_mbar_init(pb_smem(&acce[b]), 8 * PB_CTAS); }\n"
             << "        pb_mbar_init(pb_smem(&done_bar), 1);\n"
             << "#ifdef PB_TEST_STALL\n        pb_mbar_init(pb_smem(&stall_bar), 1);\n#endif\n"
             << "        asm volatile(\"fence.mbarrier_init.release.cluster;\" ::: \"memory\");\n"
             << "    }\n"
             // Warp 9 of each CTA allocates (a pair allocates together,
             // the same columns in both CTAs).
             << "    if (warp == 9) {\n"
             << "        asm volatile(\"tcgen05.alloc.cta_group::" << ctas << ".sync.aligned.shared::cta.b32 [%0], 512;\" :: \"r\"(pb_smem(&tmem_slot)) : \"memory\");\n"
             << "        asm volatile(\"tcgen05.relinquish_alloc_permit.cta_group::" << ctas << ".sync.aligned;\" ::: \"memory\");\n"
             << "    }\n"
             << "    asm volatile(\"tcgen05.fence::before_thread_sync;\" ::: \"memory\");\n"
             << (pair ? "    pb_cluster_sync();  // barriers initialised and TMEM allocated in both CTAs\n"
                      : "    __syncthreads();\n")
             << "    asm volatile(\"tcgen05.fence::after_thread_sync;\" ::: \"memory\");\n"
             << "    const pb_u32 tmem = tmem_slot;\n"
             << "    const int num_kb = " << (pair ? kb_unit / 2 : kb_unit) << ";  // k-blocks per work unit\n"
             << "    const int periods = (num_kb + PB_PERIOD - 1) / PB_PERIOD;  // the last may be partial\n"
             << "    if (warp == 8) {\n"
             << "        if (lane == 0) {\n"
             // producer
             << "            int g = 0;\n"
             << "            bool stop = false;\n"
             << "            for (pb_u32 t = blockIdx.x / PB_CTAS; t < tiles && !stop; t += gridDim.x / PB_CTAS) {\n"
             << "                int m0, n0;\n"
             << "                pb_u32 bt;\n"
             << "                pb_tile_origin(t / PB_SPLIT, m0, n0, bt);\n"
             << "                m0 += (int)(rank * PB_BM);   // this CTA's rows of A\n"
             << "                n0 += (int)(rank * PB_BNH);  // and of B (N)\n"
             << (nb > 1 ? "                m0 += (int)(bt * " + std::to_string(M) + "u);  // batch bt's rows of the stacked halves\n"
                          "                n0 += (int)(bt * " + std::to_string(N) + "u);\n"
                        : std::string{})
             << "                const int kbase = (int)(t % PB_SPLIT) * num_kb;\n"
             << "                for (int kb = 0; kb < num_kb; ++kb, ++g) {\n"
             << "                    const int s = g % PB_STAGES;\n"
             << "                    const pb_u32 phase = (pb_u32)(g / PB_STAGES) & 1u;\n"
             << "                    if (!pb_wait(pb_smem(&empty_bar[s]), phase ^ 1u, &abort_flag, err, 1)) { stop = true; break; }\n"
             << "                    const pb_u32 st = base + (pb_u32)s * PB_STAGE_BYTES;\n"
             << (pair ? "                    const pb_u32 fb = pb_mapa(pb_smem(&full_bar[s]), 0u);\n"
                        "                    if (rank == 0) pb_mbar_expect_tx(pb_smem(&full_bar[s]), 2 * PB_STAGE_BYTES);\n"
                      : "                    const pb_u32 fb = pb_smem(&full_bar[s]);\n"
                        "                    pb_mbar_expect_tx(fb, PB_STAGE_BYTES);\n")
             << "                    const int kx = (kbase + kb) * PB_BK;\n"
             << "                    pb_tma_load(st, &tm_ahi, fb, kx, m0);\n"
             << "                    pb_tma_load(st + PB_TILE_A_BYTES, &tm_alo, fb, kx, m0);\n"
             << "                    pb_tma_load(st + 2 * PB_TILE_A_BYTES, &tm_bhi, fb, kx, n0);\n"
             << "                    pb_tma_load(st + 2 * PB_TILE_A_BYTES + PB_TILE_B_BYTES, &tm_blo, fb, kx, n0);\n"
             << "                    issued = g + 1;\n"
             << "                }\n"
             << "            }\n"
             << "        }\n"
             << "        __syncwarp();\n"
             << "    } else if (warp == 9) {\n"
             << "        if (lane == 0 && rank == 0) {\n"
             // MMA issuer: period p (PB_PERIOD k-blocks, never straddling a
             // tile) accumulates from zero into TMEM buffer p % 2 (columns
             // 256 (p % 2)..+255); before reusing a buffer it waits for the
             // drain of period p - 2.
             << "            int g = 0, per_base = 0;\n"
             << "            bool stop = false;\n"
             // Failure-detection test hook: CTA 0 waits on a barrier nothing
             // arrives on, so its bounded wait gives up (site 7).
             << "#ifdef PB_TEST_STALL\n"
             // Half the usual budget, so that this wait is the first to give up.
             << "            if (blockIdx.x == 0u && !pb_wait_for(pb_smem(&stall_bar), 0u, &abort_flag, err, 7, PB_WAIT_CYCLES / 2)) stop = true;\n"
             << "#endif\n"
             << "            for (pb_u32 t = blockIdx.x / PB_CTAS; t < tiles && !stop; t += gridDim.x / PB_CTAS, per_base += periods) {\n"
             << "                for (int kb = 0; kb < num_kb; ++kb, ++g) {\n"
             << "                    const int s = g % PB_STAGES;\n"
             << "                    const pb_u32 phase = (pb_u32)(g / PB_STAGES) & 1u;\n"
             << "                    const int per = per_base + kb / PB_PERIOD, pos = kb % PB_PERIOD;\n"
             << "                    const pb_u32 buf = (pb_u32)per & 1u;\n"
             << "                    if (pos == 0 && per >= 2) {\n"
             << "                        if (!pb_wait(pb_smem(&acce[buf]), (pb_u32)((per >> 1) - 1) & 1u, &abort_flag, err, 6)) { stop = true; break; }\n"
             << "                        asm volatile(\"tcgen05.fence::after_thread_sync;\" ::: \"memory\");\n"
             << "                    }\n"
             << "                    if (!pb_wait(pb_smem(&full_bar[s]), phase, &abort_flag, err, 2)) { stop = true; break; }\n"
             << "                    consumed = g + 1;\n"
             << "                    asm volatile(\"tcgen05.fence::after_thread_sync;\" ::: \"memory\");\n"
             << "                    const pb_u32 st = base + (pb_u32)s * PB_STAGE_BYTES;\n"
             << "                    const pb_u32 d = tmem + buf * (pb_u32)PB_BN;\n"
             << "                    #pragma unroll\n"
             << "                    for (int kk = 0; kk < PB_BK / 8; ++kk) {\n"
             << "                        const pb_u64 ahi = pb_desc(st + kk * 32);\n"
             << "                        const pb_u64 alo = pb_desc(st + PB_TILE_A_BYTES + kk * 32);\n"
             << "                        const pb_u64 bhi = pb_desc(st + 2 * PB_TILE_A_BYTES + kk * 32);\n"
             << "                        const pb_u64 blo = pb_desc(st + 2 * PB_TILE_A_BYTES + PB_TILE_B_BYTES + kk * 32);\n"
             << "                        pb_mma(d, ahi, bhi, (pos | kk) != 0);\n"
             << "                        pb_mma(d, ahi, blo, 1u);\n"
             << "                        pb_mma(d, alo, bhi, 1u);\n"
             << "                    }\n"
             << "                    pb_commit(pb_smem(&empty_bar[s]));\n"
             << "                    if (pos == PB_PERIOD - 1 || kb == num_kb - 1) pb_commit(pb_smem(&accf[buf]));\n"
             << "                }\n"
             << "            }\n"
             // Whether or not the loops finished: completes once every MMA
             // issued so far has (the teardown waits for it).
             << "            pb_commit_local(pb_smem(&done_bar));\n"
             << "        }\n"
             << "        __syncwarp();\n"
             << "    } else {\n"
             // drain + epilogue warps
             << "        const pb_u32 quad = warp & 3u, half = warp >> 2;\n"
             << "        int per = 0;\n"
             << "        bool ok = true;\n"
             << "        for (pb_u32 t = blockIdx.x / PB_CTAS; t < tiles && ok; t += gridDim.x / PB_CTAS) {\n"
             << "            int m0, n0;\n"
             << "            pb_u32 bt;\n"
             << "            pb_tile_origin(t / PB_SPLIT, m0, n0, bt);\n"
             << "            m0 += (int)(rank * PB_BM);  // this CTA's 128 rows of the tile\n"
             << batch_ptrs
             << "            float acc[PB_BN / 2];\n"
             << "            #pragma unroll\n"
             << "            for (int j = 0; j < PB_BN / 2; ++j) acc[j] = 0.0f;\n"
             << "            for (int q = 0; q < periods; ++q, ++per) {\n"
             << "                const pb_u32 buf = (pb_u32)per & 1u;\n"
             << "                ok = __all_sync(0xffffffffu, pb_wait(pb_smem(&accf[buf]), (pb_u32)(per >> 1) & 1u, &abort_flag, err, 3) && !abort_flag);\n"
             << "                if (!ok) break;\n"
             << "                asm volatile(\"tcgen05.fence::after_thread_sync;\" ::: \"memory\");\n"
             << "                const pb_u32 taddr = tmem + ((quad * 32u) << 16) + buf * (pb_u32)PB_BN + half * (pb_u32)(PB_BN / 2);\n"
             << "                #pragma unroll\n"
             << "                for (int c = 0; c < PB_BN / 64; ++c) {\n"
             << "                    pb_u32 v[32];\n"
             << "                    PB_TMEM_LD32(taddr + (pb_u32)(c * 32), v);\n"
             << "                    asm volatile(\"tcgen05.wait::ld.sync.aligned;\" ::: \"memory\");\n"
             << "                    #pragma unroll\n"
             << "                    for (int j = 0; j < 32; ++j) acc[c * 32 + j] = acc[c * 32 + j] + __uint_as_float(v[j]);\n"
             << "                }\n"
             << "                asm volatile(\"tcgen05.fence::before_thread_sync;\" ::: \"memory\");\n"
             << "                __syncwarp();\n"
             << (pair ? "                if (lane == 0) pb_mbar_arrive_cl(pb_mapa(pb_smem(&acce[buf]), 0u));\n"
                      : "                if (lane == 0) pb_mbar_arrive(pb_smem(&acce[buf]));\n")
             << "            }\n"
             << (softmax && !softmax_split ? "            // The softmax epilogue exchanges row statistics between the\n"
                           "            // column halves: all 256 drain threads agree on going on.\n"
                           "            ok = pb_bar_all(ok);\n" : "")
             << "            if (!ok) break;\n"
             << "            const int r = m0 + (int)(quad * 32u + lane);\n"
             << "            const pb_u64 rr = (pb_u64)r;\n"
             << "            (void)rr;\n";
        // Leaf loads by column stride: 1 and 16-byte aligned -> float4 per
        // 4 columns; 0 -> one load per row, hoisted out of the column loops;
        // otherwise one scalar per element.
        // With N not a multiple of 4 a group of four columns can cross the
        // end of a row: scalar loads, each behind a column check.
        const bool vec_n = N % 4 == 0;
        const int64_t Np = (N + 3) / 4 * 4;  // row pitch of the split-K partials
        std::vector<int> leaf_mode(order.size());
        for (size_t li = 0; li < order.size(); ++li) {
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            const int64_t sr = v.map.st[0], sc = v.map.st[1];
            if (sc == 0)
                leaf_mode[li] = 0;
            else if (vec_n && sc == 1 && v.map.off % 4 == 0 && sr % 4 == 0)
                leaf_mode[li] = 1;
            else
                leaf_mode[li] = 2;
        }
        // Emits the fused epilogue of one float4 of outputs at row `rr`,
        // columns cc..cc+3: y[e] = pb_e0(value(e), leaves at (rr, cc + e)).
        std::vector<std::string> cvar = {"rr", "cc"};
        std::vector<std::string> evar = {"rr", "ce"};
        auto emit_epilogue4 = [&](std::ostringstream& os, const std::string& ind, const std::string& value) {
            for (size_t li = 0; li < order.size(); ++li) {
                if (leaf_mode[li] != 1) continue;
                const vnode& v = b.nodes[static_cast<size_t>(order[li])];
                os << ind << "const float4 q" << li << " = pb_ld4(in" << v.buffer << " + "
                   << address(v.map, cvar, true, -1) << ");\n";
            }
            os << ind << "float y[4];\n" << ind << "#pragma unroll\n" << ind << "for (int e = 0; e < 4; ++e) {\n"
               << ind << "    const pb_u64 ce = cc + (pb_u64)e;\n" << ind << "    (void)ce;\n";
            if (!vec_n) os << ind << "    y[e] = 0.0f;\n" << ind << "    if (ce >= " << N << "ull) continue;\n";
            for (size_t li = 0; li < order.size(); ++li) {
                const vnode& v = b.nodes[static_cast<size_t>(order[li])];
                if (leaf_mode[li] == 0)
                    os << ind << "    const float x" << li << " = h" << li << ";\n";
                else if (leaf_mode[li] == 1)
                    os << ind << "    const float x" << li << " = e == 0 ? q" << li << ".x : e == 1 ? q" << li
                       << ".y : e == 2 ? q" << li << ".z : q" << li << ".w;\n";
                else
                    os << ind << "    const float x" << li << " = pb_ld(in" << v.buffer << " + "
                       << address(v.map, evar, true, -1) << ");\n";
            }
            os << ind << "    y[e] = pb_e0(" << value;
            for (size_t li = 0; li < order.size(); ++li) os << ", x" << li;
            os << ");\n" << ind << "}\n";
        };
        auto emit_hoisted = [&](std::ostringstream& os, const std::string& ind) {
            for (size_t li = 0; li < order.size(); ++li) {
                if (leaf_mode[li] != 0) continue;
                const vnode& v = b.nodes[static_cast<size_t>(order[li])];
                std::vector<std::string> cv = {"rr", "0"};
                os << ind << "const float h" << li << " = pb_ld(in" << v.buffer << " + " << address(v.map, cv, true, 1)
                   << ");\n";
            }
        };
        if (softmax && !softmax_split) {
            // Softmax over the output row, per tile: y = tree(acc) (columns
            // past N count as -inf), m = the tile row's maximum (the two
            // column halves meet in shared memory), E = exp(y - m) stored in
            // place of y, and (m, sum E) stored per (row, column tile) for
            // the normalising pass.
            body << "            const float pb_ninf = __int_as_float(0xff800000);\n"
                 << "            float mx = pb_ninf;\n"
                 << "            if (rr < " << M << "ull) {\n";
            emit_hoisted(body, "            ");
            body << "            #pragma unroll\n"
                 << "            for (int c = 0; c < PB_BN / 64; ++c) {\n"
                 << "                const int cbase = n0 + (int)half * (PB_BN / 2) + c * 32;\n"
                 << "                #pragma unroll\n"
                 << "                for (int j = 0; j < 32; j += 4) {\n"
                 << "                    const pb_u64 cc = (pb_u64)(cbase + j);\n"
                 << "                    if (cc >= " << N << "ull) {\n"
                 << "                        acc[c * 32 + j] = pb_ninf; acc[c * 32 + j + 1] = pb_ninf;\n"
                 << "                        acc[c * 32 + j + 2] = pb_ninf; acc[c * 32 + j + 3] = pb_ninf;\n"
                 << "                        continue;\n"
                 << "                    }\n";
            emit_epilogue4(body, "                    ", "acc[c * 32 + j + e]");
            body << "                    #pragma unroll\n"
                 << "                    for (int e = 0; e < 4; ++e) acc[c * 32 + j + e] = cc + (pb_u64)e < " << N
                 << "ull ? y[e] : pb_ninf;\n"
                 << "                }\n"
                 << "            }\n"
                 << "            #pragma unroll\n"
                 << "            for (int j = 0; j < PB_BN / 2; ++j) mx = acc[j] > mx ? acc[j] : mx;\n"
                 << "            }\n"
                 << "            const pb_u32 row = quad * 32u + lane;\n"
                 << "            sm_max[half][row] = mx;\n"
                 << "            pb_bar_drain();\n"
                 << "            mx = sm_max[0][row] > sm_max[1][row] ? sm_max[0][row] : sm_max[1][row];\n"
                 << "            float sum = 0.0f;\n"
                 << "            if (rr < " << M << "ull) {\n"
                 << "            #pragma unroll\n"
                 << "            for (int j = 0; j < PB_BN / 2; ++j) {\n"
                 << "                const float e = __expf(acc[j] - mx);\n"
                 << "                acc[j] = e;\n"
                 << "                sum = sum + e;\n"
                 << "            }\n"
                 << "            }\n"
                 << "            sm_sum[half][row] = sum;\n"
                 << "            pb_bar_drain();\n"
                 << "            sum = sm_sum[0][row] + sm_sum[1][row];\n"
                 << "            if (rr < " << M << "ull) {\n"
                 << "            if (half == 0u) stats[rr * " << tiles_n << "ull + (pb_u64)(n0 / PB_BN)] = make_float2(mx, sum);\n"
                 << "            #pragma unroll\n"
                 << "            for (int c = 0; c < PB_BN / 64; ++c) {\n"
                 << "                const int cbase = n0 + (int)half * (PB_BN / 2) + c * 32;\n"
                 << "                float* orow = out + rr * " << N << "ull + cbase;\n"
                 << "                #pragma unroll\n"
                 << "                for (int j = 0; j < 32; j += 4) {\n"
                 << "                    const pb_u64 cc = (pb_u64)(cbase + j);\n"
                 << "                    if (cc >= " << N << "ull) continue;\n";
            if (vec_n)
                body << "                    pb_st4(orow + j, make_float4(acc[c * 32 + j], acc[c * 32 + j + 1], "
                        "acc[c * 32 + j + 2], acc[c * 32 + j + 3]));\n";
            else
                body << "                    #pragma unroll\n"
                     << "                    for (int e = 0; e < 4; ++e) if (cc + (pb_u64)e < " << N
                     << "ull) orow[j + e] = acc[c * 32 + j + e];\n";
            body << "                }\n"
                 << "            }\n"
                 << "            }\n";
        } else if (split > 1) {
            // Raw partial tile of this K split; the split-K kernel below
            // sums the partials and applies the epilogue.
            body << "            const pb_u64 sp = (pb_u64)(t % PB_SPLIT);\n"
                 << "            if (rr < " << M << "ull) {\n"
                 << "            #pragma unroll\n"
                 << "            for (int c = 0; c < PB_BN / 64; ++c) {\n"
                 << "                const int cbase = n0 + (int)half * (PB_BN / 2) + c * 32;\n"
                 << "                float* orow = out + sp * " << M * Np << "ull + rr * " << Np << "ull + cbase;\n"
                 << "                #pragma unroll\n"
                 << "                for (int j = 0; j < 32; j += 4)\n"
                 << "                    if ((pb_u64)(cbase + j) < " << Np << "ull)\n"
                 << "                        pb_st4(orow + j, make_float4(acc[c * 32 + j], acc[c * 32 + j + 1], "
                    "acc[c * 32 + j + 2], acc[c * 32 + j + 3]));\n"
                 << "            }\n"
                 << "            }\n";
        } else if (so != nullptr) {
            // Split output: the result as the next GEMM's A operand halves,
            // hi = rn_tf32(y) and lo = rn_tf32(y - hi) in rows of N = Kp
            // floats; an Inf or NaN result sets the flag and gets lo = 0.
            body << "            if (rr < " << M << "ull) {\n";
            emit_hoisted(body, "            ");
            body << "            bool bad = false;\n"
                 << "            #pragma unroll\n"
                 << "            for (int c = 0; c < PB_BN / 64; ++c) {\n"
                 << "                const int cbase = n0 + (int)half * (PB_BN / 2) + c * 32;\n"
                 << "                float* hrow = out + rr * " << N << "ull + cbase;\n"
                 << "                float* lrow = lo_out + rr * " << N << "ull + cbase;\n"
                 << "                #pragma unroll\n"
                 << "                for (int j = 0; j < 32; j += 4) {\n"
                 << "                    const pb_u64 cc = (pb_u64)(cbase + j);\n"
                 << "                    if (cc >= " << N << "ull) continue;\n";
            emit_epilogue4(body, "                    ", "acc[c * 32 + j + e]");
            body << "                    float h[4], l[4];\n"
                 << "                    #pragma unroll\n"
                 << "                    for (int e = 0; e < 4; ++e) {\n"
                 << "                        const bool fin = isfinite(y[e]);\n"
                 << "                        bad = bad || !fin;\n"
                 << "                        h[e] = pb_tf32_hi(y[e]);\n"
                 << "                        l[e] = fin ? pb_tf32_rn(y[e] - h[e]) : 0.0f;\n"
                 << "                    }\n"
                 << "                    pb_st4(hrow + j, make_float4(h[0], h[1], h[2], h[3]));\n"
                 << "                    pb_st4(lrow + j, make_float4(l[0], l[1], l[2], l[3]));\n"
                 << "                }\n"
                 << "            }\n"
                 << "            if (bad) atomicOr(split_flag, 1);\n"
                 << "            }\n";
        } else {
            // Rows past M and columns past N (edge tiles) are neither read
            // (leaves) nor written.
            body << "            if (rr < " << M << "ull) {\n";
            emit_hoisted(body, "            ");
            body << "            #pragma unroll\n"
                 << "            for (int c = 0; c < PB_BN / 64; ++c) {\n"
                 << "                const int cbase = n0 + (int)half * (PB_BN / 2) + c * 32;\n"
                 << "                float* orow = out + rr * " << N << "ull + cbase;\n"
                 << "                #pragma unroll\n"
                 << "                for (int j = 0; j < 32; j += 4) {\n"
                 << "                    const pb_u64 cc = (pb_u64)(cbase + j);\n"
                 << "                    if (cc >= " << N << "ull) continue;\n";
            emit_epilogue4(body, "                    ", "acc[c * 32 + j + e]");
            if (vec_n)
                body << "                    pb_st4(orow + j, make_float4(y[0], y[1], y[2], y[3]));\n";
            else
                body << "                    #pragma unroll\n"
                     << "                    for (int e = 0; e < 4; ++e) if (cc + (pb_u64)e < " << N
                     << "ull) orow[j + e] = y[e];\n";
            body << "                }\n"
                 << "            }\n"
                 << "            }\n";
        }
        body
             << "        }\n"
             << "    }\n"
             // Teardown: wait (bounded, ignoring the abort flag) for the
             // commit that follows every MMA issued -- so no MMA or commit
             // arrival lands after the CTA leaves -- and, after an abort, for
             // every TMA copy issued but not consumed, so nothing writes
             // freed TMEM or shared memory.
             ;
        if (!pair)
            body << "    __syncthreads();\n"
                 << "    if (threadIdx.x == 0) {\n"
                 << "        pb_wait_quiet(pb_smem(&done_bar), 0u);\n"
                 << "        if (abort_flag)\n"
                 << "            for (int g = consumed; g < issued; ++g)\n"
                 << "                pb_wait_quiet(pb_smem(&full_bar[g % PB_STAGES]), (pb_u32)(g / PB_STAGES) & 1u);\n"
                 << "    }\n"
                 << "    asm volatile(\"tcgen05.fence::before_thread_sync;\" ::: \"memory\");\n"
                 << "    __syncthreads();\n";
        else
            // A pair: once both CTAs have left their roles (no more loads,
            // arrivals or MMAs issued), the first CTA waits for the MMAs
            // (which write both CTAs' TMEM and read both CTAs' shared
            // memory) and, after an abort, for every stage either CTA
            // loaded but no MMA consumed. The first CTA arms a stage for
            // both CTAs' bytes when it loads its own half: where only the
            // second CTA loaded, it arms the barrier for those bytes now;
            // where only it loaded, it counts the missing half as landed.
            // Either way the phase completes when the bytes that were
            // loaded have landed. Then both CTAs free the TMEM.
            body << "    asm volatile(\"tcgen05.fence::before_thread_sync;\" ::: \"memory\");\n"
                 << "    pb_cluster_sync();\n"
                 << "    if (threadIdx.x == 0 && rank == 0) {\n"
                 << "        pb_wait_quiet(pb_smem(&done_bar), 0u);\n"
                 << "        if (abort_flag) {\n"
                 << "            const int peer_issued = pb_peer_int(&issued);\n"
                 << "            const int hi = issued > peer_issued ? issued : peer_issued;\n"
                 << "            for (int g = consumed; g < hi; ++g) {\n"
                 << "                const pb_u32 fb = pb_smem(&full_bar[g % PB_STAGES]);\n"
                 << "                if (g >= issued) pb_mbar_expect_tx(fb, PB_STAGE_BYTES);\n"
                 << "                else if (g >= peer_issued) pb_mbar_complete_tx(fb, PB_STAGE_BYTES);\n"
                 << "                pb_wait_quiet(fb, (pb_u32)(g / PB_STAGES) & 1u);\n"
                 << "            }\n"
                 << "        }\n"
                 << "    }\n"
                 << "    asm volatile(\"tcgen05.fence::before_thread_sync;\" ::: \"memory\");\n"
                 << "    pb_cluster_sync();\n";
        body << "    if (warp == 9) {\n"
             << "        asm volatile(\"tcgen05.fence::after_thread_sync;\" ::: \"memory\");\n"
             << "        asm volatile(\"tcgen05.dealloc.cta_group::" << ctas << ".sync.aligned.b32 %0, 512;\" :: \"r\"(tmem) : \"memory\");\n"
             << "    }\n";
        launch_spec l;
        l.name = "pb_gemm_tc_" + hex8(src.str() + body.str());
        src << "extern \"C\" __global__ void __launch_bounds__(320, 1) " << l.name
            << "(const __grid_constant__ pb_tmap tm_ahi, const __grid_constant__ pb_tmap tm_alo, "
               "const __grid_constant__ pb_tmap tm_bhi, const __grid_constant__ pb_tmap tm_blo, ";
        const std::string gsuf = nb > 1 ? "_g" : "";
        for (size_t i = 0; i < k.leaves.size(); ++i) src << "const float* __restrict__ in" << i << gsuf << ", ";
        src << "float* __restrict__ out" << gsuf << ", " << (softmax && !softmax_split ? "float2* __restrict__ stats, " : "")
            << (so != nullptr ? "float* __restrict__ lo_out, int* __restrict__ split_flag, " : "")
            << "int* __restrict__ err, const int* __restrict__ nf) {\n" << body.str() << "}\n";
        l.source = src.str();
        l.schedule = pair ? "gemm tcgen05 3xTF32 CTA pairs (cta_group::2) 256x256x32, 3-stage TMA ring (128B swizzle, "
                            "no multicast), two TMEM accumulators drained per period into fp32 registers, fused "
                            "epilogue, grouped tile order"
                          : "gemm tcgen05 3xTF32 128x256x16, 4-stage TMA ring (64B swizzle, no multicast), "
                            "two TMEM accumulators drained per period into fp32 registers, fused epilogue, "
                            "grouped tile order";
        // Persistent CTAs (grid = SMs x resident CTAs = 148) when tiles are
        // short (K <= 4096): hiding each tile's epilogue behind the next
        // tile's first period then wins (A/B on one box: config 5's GEMM1,
        // K = 4096, 6 % fewer cycles). Longer tiles run one per CTA
        // (grid = tiles), where hardware scheduling keeps the running tiles
        // closer together in L2 (K = 8192 and 16384: 1-3 % fewer cycles than
        // persistent; CTA pairs the same: config 5's GEMM2, K = 16384, 8.66-8.79
        // ms persistent against 8.58-8.71). The kernel is the same; its tile
        // loop runs once.
        const bool persistent = kb_unit * kBK <= 4096;
        l.grid = {static_cast<uint32_t>((persistent ? std::min<int64_t>(units, slots) : units) * ctas), 1, 1};
        l.cluster_x = static_cast<uint32_t>(ctas);
        if (persistent) {
            l.persistent_units = units;
            l.schedule += ", persistent CTAs (epilogue overlaps the next tile)";
        }
        if (split > 1) l.schedule += ", split-K x" + std::to_string(split) + " (raw partial tiles)";
        if (nb > 1) l.schedule += ", " + std::to_string(nb) + " batches grouped in one launch";
        if (softmax && !softmax_split)
            l.schedule += ", softmax epilogue (exp(y - tile row max) and per-tile row (max, sum))";
        l.block = {320, 1, 1};
        const int bk = pair ? 2 * kBK : kBK;
        l.smem = (pair ? kPairStages : kStages) * (2 * kBM * bk * 4 + 2 * (kBN / ctas) * bk * 4) + 1024;
        auto tmap_arg = [&](int temp, int64_t rows, int box_rows) {
            kernel_arg a;
            a.kind = arg_kind::tmap;
            a.index = temp;
            a.value = static_cast<uint64_t>(rows);
            a.cols = Kp;
            a.box_rows = box_rows;
            a.box_cols = pair ? 2 * kBK : kBK;
            a.swizzle = pair ? 3 : 2; // 128B / 64B: the box's inner extent is one swizzle row
            return a;
        };
        l.args = {tmap_arg(a_hi, nb * M, kBM), tmap_arg(a_lo, nb * M, kBM), tmap_arg(b_hi, nb * N, kBN / ctas),
                  tmap_arg(b_lo, nb * N, kBN / ctas)};
        for (const kernel_arg& a : k.leaves) l.args.push_back(a);
        kernel_arg out_arg = temp_arg(out);
        out_arg.elem_offset = out_off;
        l.args.push_back(split > 1 ? temp_arg(part) : out_arg);
        if (softmax && !softmax_split) l.args.push_back(temp_arg(stats));
        if (so != nullptr) {
            l.args.push_back(temp_arg(so->lo));
            l.args.push_back(temp_arg(so->flag));
            l.schedule += ", split-output epilogue (the next GEMM's A operand halves)";
        }
        kernel_arg e;
        e.kind = arg_kind::error_word;
        l.args.push_back(e);
        l.args.push_back(temp_arg(nf));
        finish_kernel(l);
        p_.launches.push_back(std::move(l));
        if (split == 1) return out;

        // ---- 4b. split-K + softmax: one CTA per row sums the partials in
        // split order, applies the epilogue, and runs the row softmax (max,
        // exp(y - max), sum, one division, multiplies) on values held in
        // registers: the result is written once.
        if (softmax_split) {
            const int64_t NV = N / 1024; // float4 columns per thread
            std::ostringstream ks;
            ks << kernel_prelude() << efn;
            std::ostringstream kb;
            kb << "    if (*(const volatile int*)nf != 0) return;  // the CUDA-core GEMM writes out\n"
               << "    __shared__ float red_m[8], red_s[8];\n"
               << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n"
               << "    for (pb_u64 rr = blockIdx.x; rr < " << M << "ull; rr += gridDim.x) {\n"
               << "        float v[" << NV << "][4];\n";
            emit_hoisted(kb, "        ");
            kb << "        #pragma unroll\n"
               << "        for (int q = 0; q < " << NV << "; ++q) {\n"
               << "            const pb_u64 cc = 4u * ((pb_u64)threadIdx.x + 256u * (pb_u64)q);\n"
               << "            const pb_u64 o = rr * " << N << "ull + cc;\n"
               << "            float4 s = pb_ld4(part + o);\n"
               << "            #pragma unroll\n"
               << "            for (int p = 1; p < " << split << "; ++p) {\n"
               << "                const float4 w = pb_ld4(part + (pb_u64)p * " << M * N << "ull + o);\n"
               << "                s.x = s.x + w.x; s.y = s.y + w.y; s.z = s.z + w.z; s.w = s.w + w.w;\n"
               << "            }\n"
               << "            const float sv[4] = {s.x, s.y, s.z, s.w};\n";
            emit_epilogue4(kb, "            ", "sv[e]");
            kb << "            #pragma unroll\n"
               << "            for (int e = 0; e < 4; ++e) v[q][e] = y[e];\n"
               << "        }\n"
               << "        float m = __int_as_float(0xff800000);\n"
               << "        #pragma unroll\n"
               << "        for (int q = 0; q < " << NV << "; ++q)\n"
               << "            #pragma unroll\n"
               << "            for (int e = 0; e < 4; ++e) m = v[q][e] > m ? v[q][e] : m;\n"
               << "        #pragma unroll\n"
               << "        for (int x = 16; x > 0; x >>= 1) { const float t = __shfl_xor_sync(0xffffffffu, m, x); m = t > m ? t : m; }\n"
               << "        if (lane == 0u) red_m[warp] = m;\n"
               << "        __syncthreads();\n"
               << "        m = red_m[0];\n"
               << "        #pragma unroll\n"
               << "        for (int w = 1; w < 8; ++w) m = red_m[w] > m ? red_m[w] : m;\n"
               << "        float sum = 0.0f;\n"
               << "        #pragma unroll\n"
               << "        for (int q = 0; q < " << NV << "; ++q)\n"
               << "            #pragma unroll\n"
               << "            for (int e = 0; e < 4; ++e) { v[q][e] = __expf(v[q][e] - m); sum = sum + v[q][e]; }\n"
               << "        #pragma unroll\n"
               << "        for (int x = 16; x > 0; x >>= 1) sum = sum + __shfl_xor_sync(0xffffffffu, sum, x);\n"
               << "        if (lane == 0u) red_s[warp] = sum;\n"
               << "        __syncthreads();\n"
               << "        sum = red_s[0];\n"
               << "        #pragma unroll\n"
               << "        for (int w = 1; w < 8; ++w) sum = sum + red_s[w];\n"
               << "        const float inv = 1.0f / sum;\n"
               << "        #pragma unroll\n"
               << "        for (int q = 0; q < " << NV << "; ++q) {\n"
               << "            const pb_u64 cc = 4u * ((pb_u64)threadIdx.x + 256u * (pb_u64)q);\n"
               << "            pb_st4(out + rr * " << N << "ull + cc, make_float4(v[q][0] * inv, v[q][1] * inv, v[q][2] * inv, v[q][3] * inv));\n"
               << "        }\n"
               << "        __syncthreads();  // red_m / red_s serve the next row\n"
               << "    }\n";
            launch_spec r;
            r.name = "pb_splitk_softmax_" + hex8(ks.str() + kb.str());
            ks << "extern \"C\" __global__ void __launch_bounds__(256) " << r.name << "(";
            for (size_t i = 0; i < k.leaves.size(); ++i) ks << "const float* __restrict__ in" << i << ", ";
            ks << "const float* __restrict__ part, float* __restrict__ out, const int* __restrict__ nf) {\n"
               << kb.str() << "}\n";
            r.source = ks.str();
            r.schedule = "split-K softmax combine: " + std::to_string(split) +
                         " partials summed in split order, fused epilogue, row softmax in registers (a CTA per row)";
            r.grid = {static_cast<uint32_t>(std::min<int64_t>(M, 148 * 8)), 1, 1};
            r.block = {256, 1, 1};
            r.args = k.leaves;
            r.args.push_back(temp_arg(part));
            r.args.push_back(out_arg);
            r.args.push_back(temp_arg(nf));
            finish_kernel(r);
            p_.launches.push_back(std::move(r));
            return out;
        }

        // ---- 4. split-K: sum the partials in split order + epilogue ---------
        {
            const int64_t n4 = M * Np / 4;
            std::ostringstream ks;
            ks << kernel_prelude() << efn;
            std::ostringstream kb;
            kb << "    if (*(const volatile int*)nf != 0) return;  // the CUDA-core GEMM writes out\n";
            kb << "    for (pb_u64 i = (pb_u64)blockIdx.x * 256u + threadIdx.x; i < " << n4
               << "ull; i += (pb_u64)gridDim.x * 256u) {\n"
               << "        const pb_u64 o = 4u * i, rr = o / " << Np << "ull, cc = o % " << Np << "ull;\n"
               << "        (void)rr; (void)cc;\n"
               << "        float4 s = pb_ld4(part + o);\n"
               << "        #pragma unroll\n"
               << "        for (int p = 1; p < " << split << "; ++p) {\n"
               << "            const float4 v = pb_ld4(part + (pb_u64)p * " << M * Np << "ull + o);\n"
               << "            s.x = s.x + v.x; s.y = s.y + v.y; s.z = s.z + v.z; s.w = s.w + v.w;\n"
               << "        }\n"
               << "        const float sv[4] = {s.x, s.y, s.z, s.w};\n";
            emit_hoisted(kb, "        ");
            emit_epilogue4(kb, "        ", "sv[e]");
            if (vec_n)
                kb << "        pb_st4(out + o, make_float4(y[0], y[1], y[2], y[3]));\n    }\n";
            else
                kb << "        #pragma unroll\n        for (int e = 0; e < 4; ++e) if (cc + (pb_u64)e < " << N
                   << "ull) out[rr * " << N << "ull + cc + e] = y[e];\n    }\n";
            launch_spec r;
            r.name = "pb_splitk_" + hex8(ks.str() + kb.str());
            ks << "extern \"C\" __global__ void __launch_bounds__(256) " << r.name << "(";
            for (size_t i = 0; i < k.leaves.size(); ++i) ks << "const float* __restrict__ in" << i << ", ";
            ks << "const float* __restrict__ part, float* __restrict__ out, const int* __restrict__ nf) {\n"
               << kb.str() << "}\n";
            r.source = ks.str();
            r.schedule = "split-K combine: " + std::to_string(split) +
                         " partials summed in split order, fused epilogue";
            r.grid = {static_cast<uint32_t>(std::min<int64_t>((n4 + 255) / 256, 148 * 8)), 1, 1};
            r.block = {256, 1, 1};
            r.args = k.leaves;
            r.args.push_back(temp_arg(part));
            r.args.push_back(out_arg);
            r.args.push_back(temp_arg(nf));
            finish_kernel(r);
            p_.launches.push_back(std::move(r));
        }
        return out;
    }

} // namespace porch::detail
