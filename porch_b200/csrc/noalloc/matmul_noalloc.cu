// pb_matmul_3xtf32_noalloc: fp32 matmul C = A @ B on tcgen05 3xTF32 that
// allocates no memory (include/porch_b200.h).
//
// Who needs it: callers that cannot let a library allocate device memory,
// e.g. code running inside a custom memory arena or allocator hook, a
// framework that forbids hidden allocations while it owns the device, or a
// context where a cudaMalloc would synchronise or fail. The regular path
// (pb_materialize) takes its temporaries from the library's caching
// allocator, which calls cuMemAlloc when its cache has no block to reuse.
//
// The 3xTF32 split needs scratch for Ahi, Alo (M x K) and Bhi, Blo (N x K,
// B transposed to K-major). Here that scratch is a file-scope device array
// of fixed size, so nothing is allocated at call time:
//  - capacity: PB_NOALLOC_SCRATCH_FLOATS floats (64 MiB); a call needs
//    2 * (M*K + N*K) floats and is rejected otherwise;
//  - every GPU that loads the library holds the array until process exit;
//  - every call shares the array: calls that overlap on the GPU (other
//    streams, other threads) race on it. The split kernels overwrite all of
//    the scratch they use before the GEMM reads it, so no call depends on
//    what a previous call left there (nothing needs to start at zero except
//    the error word, which is cleared whenever it is found set).
// Per device, on the first call with that device current, the entry point
// looks up the array's device address with cudaGetSymbolAddress (the array's
// name in host code is only a host-side stand-in, never passed to a
// kernel) and raises the GEMM kernel's shared-memory limit; make the first
// call on each device outside any stream capture.
//
// Accumulation follows the library's main GEMM: the tensor core's fp32
// accumulator loses low-order bits on every MMA added into it, so the MMAs
// of each period of P k-blocks start from zero in one of two 256-column TMEM
// buffers, and eight drain warps add each finished period into per-thread
// fp32 sums (round to nearest) while the MMAs fill the other buffer. P is
// the largest power of two <= sqrt(K) / 2 within [4, 32], which keeps the
// error at about half of a sequential fp32 FMA chain's at every K.
//
// The call is synchronous: it enqueues the work on `stream`, waits for it,
// and returns PB_ERR_RUNTIME with a message if a bounded wait inside the
// GEMM gave up (recorded in a file-scope device error word).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "porch_b200.h"

namespace porch::detail {
    void set_last_error(const std::string& message);
}

namespace {

    typedef unsigned int u32;
    typedef unsigned long long u64;

    constexpr int BM = 128;
    constexpr int BN = 256;
    constexpr int BK = 16; // one 64-byte swizzle row of fp32
    constexpr int STAGES = 4;
    constexpr int TILE_A = BM * BK * 4;
    constexpr int TILE_B = BN * BK * 4;
    constexpr int STAGE = 2 * TILE_A + 2 * TILE_B;
    constexpr int SMEM = STAGES * STAGE + 1024;
    constexpr int THREADS = 320; // warps 0-7 drain, 8 loads, 9 issues MMAs
    constexpr long long WAIT_CYCLES = 4000000000ll;
    constexpr size_t PB_NOALLOC_SCRATCH_FLOATS = size_t{16} << 20; // 64 MiB

    struct __align__(64) tmap_t {
        u64 opaque[16];
    };

} // namespace

static __device__ __align__(256) float pb_noalloc_scratch[PB_NOALLOC_SCRATCH_FLOATS];
static __device__ int pb_noalloc_error[4];

namespace {

    __device__ __forceinline__ u32 smem_addr(const void* p) {
        return (u32)__cvta_generic_to_shared(p);
    }

    __device__ __forceinline__ void mbar_init(u32 bar, u32 count) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
    }

    __device__ __forceinline__ u32 mbar_try(u32 bar, u32 parity) {
        u32 ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        return ok;
    }

    __device__ bool bounded_wait(u32 bar, u32 parity, volatile int* abort_flag, bool report, int site) {
        const long long start = clock64();
        for (;;) {
            if (mbar_try(bar, parity)) return true;
            if (*abort_flag) return false;
            if (clock64() - start > WAIT_CYCLES) {
                *abort_flag = 1;
                if (report && atomicCAS(&pb_noalloc_error[0], 0, 0x7c00 + site) == 0)
                    pb_noalloc_error[1] = (int)blockIdx.x;
                return false;
            }
        }
    }

    // K-major operand tile, 64-byte swizzle: 8-row groups 512 B apart.
    __device__ __forceinline__ u64 smem_desc(u32 addr) {
        u64 d = 0;
        d |= (u64)((addr & 0x3FFFFu) >> 4);
        d |= (u64)1 << 16;
        d |= (u64)(512 >> 4) << 32;
        d |= (u64)1 << 46;
        d |= (u64)4 << 61;
        return d;
    }

    // D f32, A/B tf32, both K-major, N >> 3, M >> 4.
    constexpr u32 IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((u32)(BN >> 3) << 17) | ((u32)(BM >> 4) << 24);

    __device__ __forceinline__ void mma(u32 tmem, u64 a, u64 b, u32 accumulate) {
        asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
                     :: "r"(tmem), "l"(a), "l"(b), "r"(IDESC), "r"(accumulate) : "memory");
    }

    __device__ __forceinline__ void commit(u32 bar) {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
    }

    __device__ __forceinline__ float tf32_rn(float x) {
        u32 r;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
        return __uint_as_float(r);
    }

    __device__ __forceinline__ float tf32_hi(float x) {
        const float r = tf32_rn(x);
        return isinf(r) && !isinf(x) ? __uint_as_float(__float_as_uint(x) & 0xFFFFE000u) : r;
    }

#define PB_NA_LD32(taddr, v)                                                                     \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15," \
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"       \
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), \
                   "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), \
                   "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), \
                   "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), \
                   "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])                              \
                 : "r"(taddr))

    __global__ void __launch_bounds__(256) split_rows(const float* __restrict__ x, float* __restrict__ hi,
                                                      float* __restrict__ lo, u64 n4) {
        for (u64 i = (u64)blockIdx.x * 256u + threadIdx.x; i < n4; i += (u64)gridDim.x * 256u) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
            if (!(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w)))
                atomicOr(&pb_noalloc_error[3], 1);
            float4 h, l;
            h.x = tf32_hi(v.x); l.x = tf32_rn(v.x - h.x);
            h.y = tf32_hi(v.y); l.y = tf32_rn(v.y - h.y);
            h.z = tf32_hi(v.z); l.z = tf32_rn(v.z - h.z);
            h.w = tf32_hi(v.w); l.w = tf32_rn(v.w - h.w);
            reinterpret_cast<float4*>(hi)[i] = h;
            reinterpret_cast<float4*>(lo)[i] = l;
        }
    }

    // B [K, N] -> Bhi, Blo [N, K]
    __global__ void __launch_bounds__(256) split_transpose(const float* __restrict__ x, float* __restrict__ hi,
                                                           float* __restrict__ lo, u64 K, u64 N) {
        __shared__ float t[64][65];
        const u64 k0 = (u64)blockIdx.y * 64u, n0 = (u64)blockIdx.x * 64u;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const u32 r = threadIdx.x / 64u + 4u * u, c = threadIdx.x % 64u;
            t[r][c] = __ldg(x + (k0 + r) * N + n0 + c);
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const u32 r = threadIdx.x / 64u + 4u * u, c = threadIdx.x % 64u;
            const float v = t[c][r];
            if (!isfinite(v)) atomicOr(&pb_noalloc_error[3], 1);
            const float h = tf32_hi(v);
            const u64 o = (n0 + r) * K + k0 + c;
            hi[o] = h;
            lo[o] = tf32_rn(v - h);
        }
    }

    // One 128 x 256 output tile per CTA. The MMAs of period p (`period`
    // k-blocks) accumulate from zero into TMEM columns 256 (p % 2)..+255;
    // before reusing a buffer the MMA thread waits for the drain of period
    // p - 2. Warp w < 8 drains TMEM lanes 32 (w % 4).. (its tile rows),
    // column half w / 4, into 128 fp32 sums, then stores them.
    __global__ void __launch_bounds__(THREADS, 1) gemm(const __grid_constant__ tmap_t tm_ahi,
                                                       const __grid_constant__ tmap_t tm_alo,
                                                       const __grid_constant__ tmap_t tm_bhi,
                                                       const __grid_constant__ tmap_t tm_blo, float* __restrict__ out,
                                                       u32 tiles_m, u32 tiles_n, int num_kb, int period, u64 ldc) {
        extern __shared__ float4 dyn[];
        __shared__ __align__(8) u64 full_bar[STAGES], empty_bar[STAGES], accf[2], acce[2], done_bar;
        __shared__ u32 tmem_slot;
        __shared__ int abort_flag, issued, consumed;
        const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
        const u32 base = (smem_addr(dyn) + 1023u) & ~1023u;
        const u32 per_group = 16u * tiles_n;
        const u32 g = blockIdx.x / per_group, first_m = g * 16u;
        const u32 gm = (tiles_m - first_m) < 16u ? (tiles_m - first_m) : 16u;
        const u32 tm = first_m + (blockIdx.x % per_group) % gm;
        const u32 tn = (blockIdx.x % per_group) / gm;
        const int m0 = (int)(tm * BM), n0 = (int)(tn * BN);
        const int periods = (num_kb + period - 1) / period; // the last may be partial
        if (threadIdx.x == 0) {
            abort_flag = 0;
            issued = 0;
            consumed = 0;
            for (int s = 0; s < STAGES; ++s) {
                mbar_init(smem_addr(&full_bar[s]), 1);
                mbar_init(smem_addr(&empty_bar[s]), 1);
            }
            for (int b = 0; b < 2; ++b) {
                mbar_init(smem_addr(&accf[b]), 1);
                mbar_init(smem_addr(&acce[b]), 8);
            }
            mbar_init(smem_addr(&done_bar), 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        if (warp == 9) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" :: "r"(smem_addr(&tmem_slot)) : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const u32 tmem = tmem_slot;
        if (warp == 8) {
            if (lane == 0) {
                const tmap_t* maps[4] = {&tm_ahi, &tm_alo, &tm_bhi, &tm_blo};
                const u32 offs[4] = {0u, (u32)TILE_A, (u32)(2 * TILE_A), (u32)(2 * TILE_A + TILE_B)};
                const int ys[4] = {m0, m0, n0, n0};
                for (int kb = 0; kb < num_kb; ++kb) {
                    const int s = kb % STAGES;
                    const u32 phase = (u32)(kb / STAGES) & 1u;
                    if (!bounded_wait(smem_addr(&empty_bar[s]), phase ^ 1u, &abort_flag, true, 1)) break;
                    const u32 st = base + (u32)s * STAGE;
                    const u32 fb = smem_addr(&full_bar[s]);
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(fb), "r"(STAGE) : "memory");
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                                     :: "r"(st + offs[i]), "l"((u64)maps[i]), "r"(fb), "r"(kb * BK), "r"(ys[i]) : "memory");
                    issued = kb + 1;
                }
            }
            __syncwarp();
        } else if (warp == 9) {
            if (lane == 0) {
                for (int kb = 0; kb < num_kb; ++kb) {
                    const int s = kb % STAGES;
                    const u32 phase = (u32)(kb / STAGES) & 1u;
                    const int per = kb / period, pos = kb % period;
                    const u32 buf = (u32)per & 1u;
                    if (pos == 0 && per >= 2) {
                        if (!bounded_wait(smem_addr(&acce[buf]), (u32)((per >> 1) - 1) & 1u, &abort_flag, true, 6))
                            break;
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    }
                    if (!bounded_wait(smem_addr(&full_bar[s]), phase, &abort_flag, true, 2)) break;
                    consumed = kb + 1;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const u32 st = base + (u32)s * STAGE;
                    const u32 d = tmem + buf * (u32)BN;
#pragma unroll
                    for (int kk = 0; kk < BK / 8; ++kk) {
                        const u64 ahi = smem_desc(st + kk * 32);
                        const u64 alo = smem_desc(st + TILE_A + kk * 32);
                        const u64 bhi = smem_desc(st + 2 * TILE_A + kk * 32);
                        const u64 blo = smem_desc(st + 2 * TILE_A + TILE_B + kk * 32);
                        mma(d, ahi, bhi, (pos | kk) != 0);
                        mma(d, ahi, blo, 1u);
                        mma(d, alo, bhi, 1u);
                    }
                    commit(smem_addr(&empty_bar[s]));
                    if (pos == period - 1 || kb == num_kb - 1) commit(smem_addr(&accf[buf]));
                }
                // Completes once every MMA issued so far has (the teardown waits for it).
                commit(smem_addr(&done_bar));
            }
            __syncwarp();
        } else {
            const u32 quad = warp & 3u, half = warp >> 2;
            float acc[BN / 2];
#pragma unroll
            for (int j = 0; j < BN / 2; ++j) acc[j] = 0.0f;
            bool ok = true;
            for (int per = 0; per < periods; ++per) {
                const u32 buf = (u32)per & 1u;
                ok = __all_sync(0xffffffffu, bounded_wait(smem_addr(&accf[buf]), (u32)(per >> 1) & 1u, &abort_flag,
                                                          true, 3) && !abort_flag);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const u32 taddr = tmem + ((quad * 32u) << 16) + buf * (u32)BN + half * (u32)(BN / 2);
#pragma unroll
                for (int c = 0; c < BN / 64; ++c) {
                    u32 v[32];
                    PB_NA_LD32(taddr + (u32)(c * 32), v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int j = 0; j < 32; ++j) acc[c * 32 + j] = acc[c * 32 + j] + __uint_as_float(v[j]);
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0)
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_addr(&acce[buf])) : "memory");
            }
            if (ok) {
                const u64 r = (u64)m0 + quad * 32u + lane;
#pragma unroll
                for (int c = 0; c < BN / 64; ++c) {
                    float* orow = out + r * ldc + (u64)(n0 + (int)half * (BN / 2) + c * 32);
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(orow + j) =
                            make_float4(acc[c * 32 + j], acc[c * 32 + j + 1], acc[c * 32 + j + 2], acc[c * 32 + j + 3]);
                }
            }
        }
        // Teardown: wait (bounded, ignoring the abort flag) for the commit
        // that follows every MMA issued, and after an abort for every TMA
        // copy issued but not consumed, so nothing lands in freed TMEM or
        // shared memory after the CTA leaves.
        __syncthreads();
        if (threadIdx.x == 0) {
            volatile int never = 0;
            (void)bounded_wait(smem_addr(&done_bar), 0u, &never, false, 4);
            if (abort_flag)
                for (int kb = consumed; kb < issued; ++kb)
                    (void)bounded_wait(smem_addr(&full_bar[kb % STAGES]), (u32)(kb / STAGES) & 1u, &never, false, 5);
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (warp == 9) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" :: "r"(tmem) : "memory");
        }
    }

    // ---------------------------------------------------------- host ---
    typedef CUresult (*encode_fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    typedef CUresult (*range_fn)(CUdeviceptr*, size_t*, CUdeviceptr);

    struct device_setup {
        std::once_flag once;
        cudaError_t status = cudaSuccess;
        float* scratch = nullptr;
    };

    constexpr int kMaxDevices = 64;
    device_setup g_setup[kMaxDevices];
    encode_fn g_encode = nullptr;
    range_fn g_range = nullptr;
    std::once_flag g_driver_once;

    int fail(int status, const std::string& message) {
        porch::detail::set_last_error(message);
        return status;
    }

    int cuda_fail(cudaError_t e, const char* what) {
        return fail(PB_ERR_RUNTIME, std::string{what} + " failed: " + cudaGetErrorName(e) + ": " +
                                        cudaGetErrorString(e));
    }

    bool encode(tmap_t* m, float* base, u64 rows, u64 cols, u32 box_rows) {
        const cuuint64_t dims[2] = {cols, rows};
        const cuuint64_t strides[1] = {cols * 4};
        const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
        const cuuint32_t es[2] = {1, 1};
        return g_encode(reinterpret_cast<CUtensorMap*>(m), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims,
                        strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }

    // Accumulation period in k-blocks: the largest power of two
    // <= sqrt(K) / 2, at least 4 and at most 32.
    int period_for(int64_t k) {
        int p = 4;
        while (p < 32 && static_cast<double>(p * 2) <= std::sqrt(static_cast<double>(k)) / 2.0) p *= 2;
        return p;
    }

    // An operand must be device (or managed) memory of the current device,
    // and `bytes` from `p` must lie inside one allocation: a host pointer, a
    // pointer into another GPU's memory or a too-short buffer would make the
    // kernels fault instead of returning an error.
    int check_operand(const void* p, size_t bytes, int device, const char* name) {
        cudaPointerAttributes attr{};
        const cudaError_t e = cudaPointerGetAttributes(&attr, p);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            return fail(PB_ERR_INVALID_ARGUMENT, std::string{"pb_matmul_3xtf32_noalloc: "} + name +
                                                     " is not a pointer the CUDA runtime knows");
        }
        if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
            return fail(PB_ERR_INVALID_ARGUMENT,
                        std::string{"pb_matmul_3xtf32_noalloc: "} + name + " must be device memory");
        if (attr.device != device)
            return fail(PB_ERR_INVALID_ARGUMENT, std::string{"pb_matmul_3xtf32_noalloc: "} + name +
                                                     " is on device " + std::to_string(attr.device) +
                                                     ", not the current device " + std::to_string(device));
        if (attr.type == cudaMemoryTypeDevice && g_range != nullptr) {
            CUdeviceptr base = 0;
            size_t size = 0;
            if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(p)) == CUDA_SUCCESS) {
                const u64 end = static_cast<u64>(base) + size;
                if (reinterpret_cast<u64>(p) + bytes > end)
                    return fail(PB_ERR_INVALID_ARGUMENT, std::string{"pb_matmul_3xtf32_noalloc: "} + name +
                                                             " is shorter than its shape needs");
            }
        }
        return PB_OK;
    }

} // namespace

extern "C" int pb_matmul_3xtf32_noalloc(const float* a, const float* b, float* c, int64_t m, int64_t n,
                                        int64_t k, void* stream) {
    if (a == nullptr || b == nullptr || c == nullptr)
        return fail(PB_ERR_INVALID_ARGUMENT, "pb_matmul_3xtf32_noalloc: a, b and c must be device pointers");
    if (m <= 0 || n <= 0 || k <= 0 || m % BM != 0 || n % BN != 0 || k % 64 != 0)
        return fail(PB_ERR_INVALID_ARGUMENT,
                    "pb_matmul_3xtf32_noalloc: needs M % 128 == 0, N % 256 == 0 and K % 64 == 0");
    // Each extent on its own first, so that the products below cannot wrap.
    const u64 cap = PB_NOALLOC_SCRATCH_FLOATS;
    const u64 need = (static_cast<u64>(m) > cap || static_cast<u64>(n) > cap || static_cast<u64>(k) > cap)
                         ? ~0ull
                         : 2ull * (static_cast<u64>(m) * static_cast<u64>(k) + static_cast<u64>(n) * static_cast<u64>(k));
    if (need > cap) {
        char msg[256];
        std::snprintf(msg, sizeof msg,
                      "pb_matmul_3xtf32_noalloc: needs 2*(M*K + N*K) floats of scratch (M=%lld N=%lld K=%lld); "
                      "the fixed array holds %llu (64 MiB)",
                      static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k), cap);
        return fail(PB_ERR_INVALID_ARGUMENT, msg);
    }
    // A is read and C written 16 bytes at a time.
    if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(c)) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(b) & 3u) != 0)
        return fail(PB_ERR_INVALID_ARGUMENT,
                    "pb_matmul_3xtf32_noalloc: a and c must be 16-byte aligned and b 4-byte aligned");
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (device < 0 || device >= kMaxDevices) return fail(PB_ERR_INVALID_ARGUMENT, "device ordinal out of range");

    std::call_once(g_driver_once, [] {
        cudaDriverEntryPointQueryResult q{};
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<encode_fn>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_range = reinterpret_cast<range_fn>(fn);
    });
    if (g_encode == nullptr) return fail(PB_ERR_RUNTIME, "cuTensorMapEncodeTiled is not available");

    const u64 mu = static_cast<u64>(m), nu = static_cast<u64>(n), ku = static_cast<u64>(k);
    int st = check_operand(a, mu * ku * 4, device, "a");
    if (st == PB_OK) st = check_operand(b, ku * nu * 4, device, "b");
    if (st == PB_OK) st = check_operand(c, mu * nu * 4, device, "c");
    if (st != PB_OK) return st;

    // Once per device, with that device current: the scratch array's device
    // address and the GEMM's shared-memory limit.
    device_setup& setup = g_setup[device];
    std::call_once(setup.once, [&] {
        void* p = nullptr;
        setup.status = cudaGetSymbolAddress(&p, pb_noalloc_scratch);
        if (setup.status != cudaSuccess) return;
        setup.scratch = static_cast<float*>(p);
        setup.status = cudaFuncSetAttribute(gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    });
    if (setup.status != cudaSuccess) return cuda_fail(setup.status, "scratch set-up");

    float* ahi = setup.scratch;
    float* alo = ahi + mu * ku;
    float* bhi = alo + mu * ku;
    float* blo = bhi + nu * ku;
    tmap_t maps[4];
    if (!encode(&maps[0], ahi, mu, ku, BM) || !encode(&maps[1], alo, mu, ku, BM) ||
        !encode(&maps[2], bhi, nu, ku, BN) || !encode(&maps[3], blo, nu, ku, BN))
        return fail(PB_ERR_RUNTIME, "cuTensorMapEncodeTiled failed");

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const u64 n4 = mu * ku / 4;
    const unsigned rows_grid = (unsigned)((n4 + 255) / 256 < 148 * 16 ? (n4 + 255) / 256 : 148 * 16);
    split_rows<<<rows_grid, 256, 0, s>>>(a, ahi, alo, n4);
    split_transpose<<<dim3((unsigned)(nu / 64), (unsigned)(ku / 64)), 256, 0, s>>>(b, bhi, blo, ku, nu);
    const u32 tiles_m = (u32)(mu / BM), tiles_n = (u32)(nu / BN);
    gemm<<<tiles_m * tiles_n, THREADS, SMEM, s>>>(maps[0], maps[1], maps[2], maps[3], c, tiles_m, tiles_n,
                                                  (int)(ku / BK), period_for(k), nu);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    int err[4] = {0, 0, 0, 0};
    e = cudaMemcpyFromSymbolAsync(err, pb_noalloc_error, sizeof err, 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "reading the error word");
    if (err[0] != 0 || err[3] != 0) {
        const int zero[4] = {0, 0, 0, 0};
        (void)cudaMemcpyToSymbolAsync(pb_noalloc_error, zero, sizeof zero, 0, cudaMemcpyHostToDevice, s);
        (void)cudaStreamSynchronize(s);
        if (err[0] == 0)
            return fail(PB_ERR_INVALID_ARGUMENT,
                        "pb_matmul_3xtf32_noalloc: A or B holds Inf or NaN, which the 3xTF32 "
                        "expansion cannot carry (an Inf high part times a zero low part is NaN); "
                        "pb_materialize handles them with an fp32 FMA chain");
        char msg[160];
        std::snprintf(msg, sizeof msg, "pb_matmul_3xtf32_noalloc: a bounded wait gave up (code %#x, block %d)",
                      err[0], err[1]);
        return fail(PB_ERR_RUNTIME, msg);
    }
    return PB_OK;
}
