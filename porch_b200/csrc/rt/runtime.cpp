// porch_b200 runtime: implementation of include/porch_b200_rt.h.
//
// Design (B200-first, not a translation of the reference's cuda_jit.cpp):
//  - libcuda / libnvrtc / libnccl are dlopen'ed once per process and their
//    entry points kept in function tables (the reference re-dlopens NVRTC on
//    every cache miss and on every is_available() call,
//    src/cuda_jit.cpp:634-660).
//  - One retained primary context per device (the reference creates a private
//    context on device 0 only, src/cuda_jit.cpp:446-455). Sharing the primary
//    context lets porch buffers interoperate with other runtime-API users in
//    the same process (NCCL, PyTorch).
//  - One non-blocking stream per (thread, device).
//  - The default memory pool of every device keeps freed blocks cached.
//  - NVRTC compiles straight to sm_100a cubin; images are cached by a 64-bit
//    hash of (source, options) and, optionally, on disk under
//    $PORCH_B200_CACHE_DIR. Modules are loaded once per (device, key) instead
//    of cuModuleLoadData on every launch (src/cuda_jit.cpp:819-823).
//  - No global driver mutex around launches: the driver API is thread safe,
//    and the only shared state here (caches) is guarded by its own mutexes.
#include "porch_b200_rt.h"

#include <cuda.h>
#include <dlfcn.h>
#include <unistd.h>
#include <nccl.h>
#include <nvrtc.h>

#include <algorithm>
#include <atomic>
#include <type_traits>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace {

// ---------------------------------------------------------------- errors --
thread_local std::string tl_error;

int fail(int status, std::string message) {
    tl_error = std::move(message);
    return status;
}

struct dl_handle {
    void* handle = nullptr;
    void* sym(const char* name) const {
        return handle ? dlsym(handle, name) : nullptr;
    }
};

dl_handle open_first(std::initializer_list<const char*> names) {
    for (const char* name : names) {
        void* h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
        if (h != nullptr) return {h};
    }
    return {};
}

// ------------------------------------------------------ driver table --
#define PB_DRIVER_FUNCTIONS(X)                                               \
    X(cuInit, CUresult (*)(unsigned int))                                    \
    X(cuDriverGetVersion, CUresult (*)(int*))                                \
    X(cuDeviceGetCount, CUresult (*)(int*))                                  \
    X(cuDeviceGet, CUresult (*)(CUdevice*, int))                             \
    X(cuDeviceGetAttribute, CUresult (*)(int*, CUdevice_attribute, CUdevice)) \
    X(cuDeviceGetName, CUresult (*)(char*, int, CUdevice))                   \
    X(cuDevicePrimaryCtxRetain, CUresult (*)(CUcontext*, CUdevice))          \
    X(cuCtxSetCurrent, CUresult (*)(CUcontext))                              \
    X(cuStreamCreate, CUresult (*)(CUstream*, unsigned int))                 \
    X(cuStreamDestroy_v2, CUresult (*)(CUstream))                            \
    X(cuStreamSynchronize, CUresult (*)(CUstream))                           \
    X(cuStreamWaitEvent, CUresult (*)(CUstream, CUevent, unsigned int))      \
    X(cuEventCreate, CUresult (*)(CUevent*, unsigned int))                   \
    X(cuEventDestroy_v2, CUresult (*)(CUevent))                              \
    X(cuEventRecord, CUresult (*)(CUevent, CUstream))                        \
    X(cuEventSynchronize, CUresult (*)(CUevent))                             \
    X(cuEventQuery, CUresult (*)(CUevent))                                   \
    X(cuEventElapsedTime, CUresult (*)(float*, CUevent, CUevent))            \
    X(cuMemAllocAsync, CUresult (*)(CUdeviceptr*, size_t, CUstream))         \
    X(cuMemAlloc_v2, CUresult (*)(CUdeviceptr*, size_t))                     \
    X(cuMemFree_v2, CUresult (*)(CUdeviceptr))                               \
    X(cuMemFreeAsync, CUresult (*)(CUdeviceptr, CUstream))                   \
    X(cuDeviceGetDefaultMemPool, CUresult (*)(CUmemoryPool*, CUdevice))      \
    X(cuMemPoolSetAttribute,                                                 \
      CUresult (*)(CUmemoryPool, CUmemPool_attribute, void*))                \
    X(cuMemHostAlloc, CUresult (*)(void**, size_t, unsigned int))            \
    X(cuMemFreeHost, CUresult (*)(void*))                                    \
    X(cuMemcpyHtoDAsync_v2,                                                  \
      CUresult (*)(CUdeviceptr, const void*, size_t, CUstream))              \
    X(cuMemcpyDtoHAsync_v2,                                                  \
      CUresult (*)(void*, CUdeviceptr, size_t, CUstream))                    \
    X(cuMemcpyDtoDAsync_v2,                                                  \
      CUresult (*)(CUdeviceptr, CUdeviceptr, size_t, CUstream))              \
    X(cuMemcpyPeerAsync, CUresult (*)(CUdeviceptr, CUcontext, CUdeviceptr,   \
                                      CUcontext, size_t, CUstream))          \
    X(cuMemsetD32Async,                                                      \
      CUresult (*)(CUdeviceptr, unsigned int, size_t, CUstream))             \
    X(cuDeviceCanAccessPeer, CUresult (*)(int*, CUdevice, CUdevice))         \
    X(cuCtxEnablePeerAccess, CUresult (*)(CUcontext, unsigned int))          \
    X(cuModuleLoadData, CUresult (*)(CUmodule*, const void*))                \
    X(cuModuleGetFunction, CUresult (*)(CUfunction*, CUmodule, const char*)) \
    X(cuFuncSetAttribute,                                                    \
      CUresult (*)(CUfunction, CUfunction_attribute, int))                   \
    X(cuFuncGetAttribute,                                                    \
      CUresult (*)(int*, CUfunction_attribute, CUfunction))                  \
    X(cuOccupancyMaxActiveBlocksPerMultiprocessor,                           \
      CUresult (*)(int*, CUfunction, int, size_t))                           \
    X(cuOccupancyMaxActiveClusters,                                          \
      CUresult (*)(int*, CUfunction, const CUlaunchConfig*))                 \
    X(cuLaunchKernelEx, CUresult (*)(const CUlaunchConfig*, CUfunction,      \
                                     void**, void**))                        \
    X(cuTensorMapEncodeTiled,                                                \
      CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,     \
                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,  \
                   const cuuint32_t*, CUtensorMapInterleave,                 \
                   CUtensorMapSwizzle, CUtensorMapL2promotion,               \
                   CUtensorMapFloatOOBfill))                                 \
    X(cuGetErrorName, CUresult (*)(CUresult, const char**))                  \
    X(cuGetErrorString, CUresult (*)(CUresult, const char**))

struct driver_api {
#define PB_DECLARE(name, type) std::type_identity_t<type> name = nullptr;
    PB_DRIVER_FUNCTIONS(PB_DECLARE)
#undef PB_DECLARE
};

#define PB_NVRTC_FUNCTIONS(X)                                                \
    X(nvrtcVersion, nvrtcResult (*)(int*, int*))                             \
    X(nvrtcCreateProgram,                                                    \
      nvrtcResult (*)(nvrtcProgram*, const char*, const char*, int,          \
                      const char* const*, const char* const*))               \
    X(nvrtcCompileProgram, nvrtcResult (*)(nvrtcProgram, int, const char* const*)) \
    X(nvrtcGetCUBINSize, nvrtcResult (*)(nvrtcProgram, size_t*))             \
    X(nvrtcGetCUBIN, nvrtcResult (*)(nvrtcProgram, char*))                   \
    X(nvrtcGetPTXSize, nvrtcResult (*)(nvrtcProgram, size_t*))               \
    X(nvrtcGetPTX, nvrtcResult (*)(nvrtcProgram, char*))                     \
    X(nvrtcGetProgramLogSize, nvrtcResult (*)(nvrtcProgram, size_t*))        \
    X(nvrtcGetProgramLog, nvrtcResult (*)(nvrtcProgram, char*))              \
    X(nvrtcDestroyProgram, nvrtcResult (*)(nvrtcProgram*))                   \
    X(nvrtcGetErrorString, const char* (*)(nvrtcResult))

struct nvrtc_api {
#define PB_DECLARE(name, type) std::type_identity_t<type> name = nullptr;
    PB_NVRTC_FUNCTIONS(PB_DECLARE)
#undef PB_DECLARE
};

#define PB_NCCL_FUNCTIONS(X)                                                 \
    X(ncclGetUniqueId, ncclResult_t (*)(ncclUniqueId*))                      \
    X(ncclCommInitAll, ncclResult_t (*)(ncclComm_t*, int, const int*))       \
    X(ncclCommInitRankConfig, ncclResult_t (*)(ncclComm_t*, int,             \
                                               ncclUniqueId, int,            \
                                               ncclConfig_t*))               \
    X(ncclCommDestroy, ncclResult_t (*)(ncclComm_t))                         \
    X(ncclCommFinalize, ncclResult_t (*)(ncclComm_t))                        \
    X(ncclCommAbort, ncclResult_t (*)(ncclComm_t))                           \
    X(ncclCommGetAsyncError, ncclResult_t (*)(ncclComm_t, ncclResult_t*))    \
    X(ncclGroupStart, ncclResult_t (*)())                                    \
    X(ncclGroupEnd, ncclResult_t (*)())                                      \
    X(ncclAllGather, ncclResult_t (*)(const void*, void*, size_t,            \
                                      ncclDataType_t, ncclComm_t,            \
                                      cudaStream_t))                         \
    X(ncclSend, ncclResult_t (*)(const void*, size_t, ncclDataType_t, int,   \
                                 ncclComm_t, cudaStream_t))                  \
    X(ncclRecv, ncclResult_t (*)(void*, size_t, ncclDataType_t, int,         \
                                 ncclComm_t, cudaStream_t))                  \
    X(ncclGetErrorString, const char* (*)(ncclResult_t))

struct nccl_table {
#define PB_DECLARE(name, type) std::type_identity_t<type> name = nullptr;
    PB_NCCL_FUNCTIONS(PB_DECLARE)
#undef PB_DECLARE
};

// ---------------------------------------------------------- fault sites --
enum fault_site {
    fault_compile,
    fault_alloc,
    fault_launch,
    fault_h2d,
    fault_d2h,
    fault_nccl_init,
    fault_nccl_coll,
    fault_site_count
};
const char* const fault_site_names[fault_site_count] = {
    "compile", "alloc", "launch", "h2d", "d2h", "nccl_init", "nccl_coll"};

struct fault_state {
    std::mutex mutex;
    long countdown[fault_site_count] = {};  // 0 = disarmed
};

fault_state& faults() {
    static fault_state* state = new fault_state();
    return *state;
}

int parse_fault_spec(const char* spec) {
    fault_state& state = faults();
    std::scoped_lock lock{state.mutex};
    for (long& c : state.countdown) c = 0;
    if (spec == nullptr) return PBRT_OK;
    std::string text{spec};
    std::stringstream stream{text};
    std::string item;
    while (std::getline(stream, item, ',')) {
        if (item.empty()) continue;
        const size_t colon = item.find(':');
        const std::string site = item.substr(0, colon);
        long n = 1;
        if (colon != std::string::npos) n = std::atol(item.c_str() + colon + 1);
        bool known = false;
        for (int s = 0; s < fault_site_count; ++s) {
            if (site == fault_site_names[s]) {
                state.countdown[s] = n > 0 ? n : 1;
                known = true;
            }
        }
        if (!known) return fail(PBRT_ERR_INVALID, "unknown fault site: " + site);
    }
    return PBRT_OK;
}

// Returns true (and sets the error) when the armed fault at `site` fires.
bool fault_fires(fault_site site) {
    fault_state& state = faults();
    std::scoped_lock lock{state.mutex};
    long& c = state.countdown[site];
    if (c <= 0) return false;
    if (--c != 0) return false;
    tl_error = std::string{"injected fault at "} + fault_site_names[site];
    return true;
}

// --------------------------------------------------------- environment --
struct device_state {
    CUdevice device = 0;
    CUcontext context = nullptr;
    CUdeviceptr error_block = 0;
    bool pool_configured = false;
};

struct environment {
    dl_handle cuda_lib;
    dl_handle nvrtc_lib;
    driver_api cu;
    nvrtc_api rtc;
    bool cuda_ok = false;
    bool nvrtc_ok = false;
    bool initialized = false;
    std::atomic<bool> ready{false}; // initialised successfully
    int init_status = PBRT_OK;
    std::string init_error;
    int device_count = 0;
    std::vector<device_state> devices;
    std::mutex device_mutex;
};

std::string describe(const environment& env, CUresult r) {
    const char* name = nullptr;
    const char* desc = nullptr;
    if (env.cu.cuGetErrorName) (void)env.cu.cuGetErrorName(r, &name);
    if (env.cu.cuGetErrorString) (void)env.cu.cuGetErrorString(r, &desc);
    std::string out = name ? name : ("CUDA_ERROR_" + std::to_string(int(r)));
    if (desc) out += std::string{": "} + desc;
    return out;
}

environment& env_raw() {
    static environment* e = [] {
        auto* env = new environment();
        env->cuda_lib = open_first({"libcuda.so.1", "libcuda.so"});
        if (env->cuda_lib.handle) {
            bool all = true;
#define PB_LOAD(name, type)                                             \
    env->cu.name = reinterpret_cast<type>(env->cuda_lib.sym(#name));    \
    all = all && env->cu.name != nullptr;
            PB_DRIVER_FUNCTIONS(PB_LOAD)
#undef PB_LOAD
            env->cuda_ok = all;
        }
        env->nvrtc_lib = open_first(
            {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"});
        if (env->nvrtc_lib.handle) {
            bool all = true;
#define PB_LOAD(name, type)                                             \
    env->rtc.name = reinterpret_cast<type>(env->nvrtc_lib.sym(#name));  \
    all = all && env->rtc.name != nullptr;
            PB_NVRTC_FUNCTIONS(PB_LOAD)
#undef PB_LOAD
            env->nvrtc_ok = all;
        }
        if (const char* spec = std::getenv("PORCH_FAULT")) (void)parse_fault_spec(spec);
        return env;
    }();
    return *e;
}

// Initialise the driver once; cached status afterwards.
int ensure_init(environment*& out) {
    environment& env = env_raw();
    out = &env;
    if (env.ready.load(std::memory_order_acquire)) return PBRT_OK;
    std::scoped_lock lock{env.device_mutex};
    if (env.initialized) {
        if (env.init_status != PBRT_OK) tl_error = env.init_error;
        return env.init_status;
    }
    env.initialized = true;
    auto set = [&](int status, std::string msg) {
        env.init_status = status;
        env.init_error = msg;
        tl_error = std::move(msg);
        return status;
    };
    if (!env.cuda_ok)
        return set(PBRT_ERR_UNAVAILABLE,
                   "CUDA tensor execution requires libcuda at runtime");
    CUresult r = env.cu.cuInit(0);
    if (r != CUDA_SUCCESS)
        return set(PBRT_ERR_DRIVER, "cuInit failed: " + describe(env, r));
    int count = 0;
    r = env.cu.cuDeviceGetCount(&count);
    if (r != CUDA_SUCCESS)
        return set(PBRT_ERR_DRIVER,
                   "cuDeviceGetCount failed: " + describe(env, r));
    if (count <= 0) return set(PBRT_ERR_UNAVAILABLE, "no CUDA device found");
    env.device_count = count;
    env.devices.resize(static_cast<size_t>(count));
    env.init_status = PBRT_OK;
    env.ready.store(true, std::memory_order_release);
    return PBRT_OK;
}

// Makes `device`'s primary context current on this thread.
int use_device(int device, environment*& envp) {
    int s = ensure_init(envp);
    if (s != PBRT_OK) return s;
    environment& env = *envp;
    if (device < 0 || device >= env.device_count)
        return fail(PBRT_ERR_INVALID,
                    "CUDA device ordinal " + std::to_string(device) +
                        " is not present (" + std::to_string(env.device_count) +
                        " devices)");
    device_state& d = env.devices[static_cast<size_t>(device)];
    if (d.context == nullptr) {
        std::scoped_lock lock{env.device_mutex};
        if (d.context == nullptr) {
            CUresult r = env.cu.cuDeviceGet(&d.device, device);
            if (r != CUDA_SUCCESS)
                return fail(PBRT_ERR_DRIVER, "cuDeviceGet failed: " + describe(env, r));
            CUcontext ctx = nullptr;
            r = env.cu.cuDevicePrimaryCtxRetain(&ctx, d.device);
            if (r != CUDA_SUCCESS)
                return fail(PBRT_ERR_DRIVER,
                            "cuDevicePrimaryCtxRetain failed: " + describe(env, r));
            r = env.cu.cuCtxSetCurrent(ctx);
            if (r != CUDA_SUCCESS)
                return fail(PBRT_ERR_DRIVER, "cuCtxSetCurrent failed: " + describe(env, r));
            CUmemoryPool pool = nullptr;
            if (env.cu.cuDeviceGetDefaultMemPool(&pool, d.device) == CUDA_SUCCESS) {
                cuuint64_t threshold = ~cuuint64_t{0};
                (void)env.cu.cuMemPoolSetAttribute(
                    pool, CU_MEMPOOL_ATTR_RELEASE_THRESHOLD, &threshold);
                d.pool_configured = true;
            }
            d.context = ctx;
        }
    }
    thread_local CUcontext tl_current = nullptr;
    if (tl_current != d.context) {
        CUresult r = env.cu.cuCtxSetCurrent(d.context);
        if (r != CUDA_SUCCESS)
            return fail(PBRT_ERR_DRIVER, "cuCtxSetCurrent failed: " + describe(env, r));
        tl_current = d.context;
    } else {
        // Another library in the process may have switched contexts; setting
        // the same context again is cheap and keeps us correct.
        (void)env.cu.cuCtxSetCurrent(d.context);
    }
    return PBRT_OK;
}

int check(environment& env, CUresult r, const char* operation) {
    if (r == CUDA_SUCCESS) return PBRT_OK;
    return fail(PBRT_ERR_DRIVER, std::string{operation} + " failed: " + describe(env, r));
}

// ------------------------------------------------------------- streams --
struct thread_streams {
    std::vector<CUstream> streams;
    ~thread_streams() {
        environment& env = env_raw();
        if (!env.cuda_ok) return;
        for (size_t d = 0; d < streams.size(); ++d) {
            if (streams[d] == nullptr) continue;
            // The primary context outlives the thread; drain then destroy.
            if (env.devices.size() > d && env.devices[d].context) {
                (void)env.cu.cuCtxSetCurrent(env.devices[d].context);
                (void)env.cu.cuStreamSynchronize(streams[d]);
                (void)env.cu.cuStreamDestroy_v2(streams[d]);
            }
        }
    }
};

thread_local thread_streams tl_streams;

// --------------------------------------------------------- compile cache --
struct compiled_image {
    std::string text;   // source + options, to verify hash hits
    std::string image;  // cubin bytes or PTX text (NUL-terminated)
    bool cubin = false;
};

struct module_cache {
    std::mutex mutex;
    std::unordered_map<uint64_t, std::unique_ptr<compiled_image>> images;
    std::map<std::pair<int, uint64_t>, CUmodule> modules;
    std::map<std::tuple<int, uint64_t, std::string>, CUfunction> functions;
    std::unordered_map<CUfunction, std::string> names;
};

module_cache& cache() {
    static module_cache* c = new module_cache();
    return *c;
}

uint64_t hash_bytes(uint64_t h, const void* data, size_t n) {
    // FNV-1a, 64-bit, followed by a final avalanche (splitmix64 finaliser).
    const auto* p = static_cast<const unsigned char*>(data);
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 0x100000001b3ULL;
    }
    return h;
}

uint64_t finish_hash(uint64_t h) {
    h ^= h >> 30;
    h *= 0xbf58476d1ce4e5b9ULL;
    h ^= h >> 27;
    h *= 0x94d049bb133111ebULL;
    h ^= h >> 31;
    return h;
}

std::string disk_cache_dir() {
    const char* dir = std::getenv("PORCH_B200_CACHE_DIR");
    return dir ? std::string{dir} : std::string{};
}

std::atomic<uint64_t> g_nvrtc_compiles{0};
std::atomic<uint64_t> g_disk_hits{0};

// Writes `bytes` to `path` through a private temporary name and a rename,
// so a reader (another process sharing the cache) sees the whole file or
// none of it.
bool write_file_atomically(const std::string& path, const std::string& bytes) {
    char suffix[48];
    std::snprintf(suffix, sizeof suffix, ".tmp.%d.%llx", static_cast<int>(getpid()),
                  static_cast<unsigned long long>(
                      std::hash<std::thread::id>{}(std::this_thread::get_id())));
    const std::string tmp = path + suffix;
    {
        std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
        if (!f) return false;
        f.write(bytes.data(), static_cast<std::streamsize>(bytes.size()));
        if (!f) return false;
    }
    if (std::rename(tmp.c_str(), path.c_str()) != 0) {
        (void)std::remove(tmp.c_str());
        return false;
    }
    return true;
}

// ----------------------------------------------------------- profiling --
struct launch_record {
    CUfunction function;
    int device;
    CUevent start;
    CUevent stop;
};

struct profiler {
    std::mutex mutex;
    bool enabled = false;
    std::vector<launch_record> records;
    std::vector<std::pair<int, CUevent>> free_events;
};

profiler& prof() {
    static profiler* p = new profiler();
    return *p;
}

std::atomic<uint64_t> g_launches{0};

CUevent take_event(environment& env, int device) {
    profiler& p = prof();
    {
        std::scoped_lock lock{p.mutex};
        for (size_t i = 0; i < p.free_events.size(); ++i) {
            if (p.free_events[i].first == device) {
                CUevent e = p.free_events[i].second;
                p.free_events[i] = p.free_events.back();
                p.free_events.pop_back();
                return e;
            }
        }
    }
    CUevent e = nullptr;
    if (env.cu.cuEventCreate(&e, CU_EVENT_DEFAULT) != CUDA_SUCCESS) return nullptr;
    return e;
}

// --------------------------------------------------------------- NCCL ----
struct nccl_env {
    dl_handle lib;
    nccl_table api;
    bool ok = false;
};

nccl_env& nccl() {
    static nccl_env* n = [] {
        auto* e = new nccl_env();
        e->lib = open_first({"libnccl.so.2", "libnccl.so",
                             "/usr/lib/x86_64-linux-gnu/libnccl.so.2"});
        if (e->lib.handle) {
            bool all = true;
#define PB_LOAD(name, type)                                          \
    e->api.name = reinterpret_cast<type>(e->lib.sym(#name));         \
    all = all && e->api.name != nullptr;
            PB_NCCL_FUNCTIONS(PB_LOAD)
#undef PB_LOAD
            e->ok = all;
        }
        return e;
    }();
    return *n;
}

int nccl_check(ncclResult_t r, const char* operation) {
    if (r == ncclSuccess) return PBRT_OK;
    nccl_env& n = nccl();
    std::string msg = std::string{operation} + " failed: ";
    msg += n.api.ncclGetErrorString ? n.api.ncclGetErrorString(r)
                                    : ("nccl error " + std::to_string(int(r)));
    return fail(PBRT_ERR_NCCL, msg);
}

struct comm_handle {
    ncclComm_t comm = nullptr;
    int device = 0;
    bool aborted = false;
    double timeout_s = 60.0; // bound on every host-side wait for this communicator
};

// Group nesting of the calling thread: inside a group NCCL only records the
// operations, so there is nothing to settle until the outermost group end.
thread_local int nccl_group_depth = 0;

// A non-blocking communicator may return ncclInProgress while the operation
// is still being enqueued on the host; nothing recorded on the stream after
// it is ordered behind it until the state leaves ncclInProgress. Polls that
// state with the communicator's deadline, aborting it on error or timeout.
int settle(comm_handle* h, const char* operation) {
    nccl_env& n = nccl();
    const auto deadline = std::chrono::steady_clock::now() +
                          std::chrono::duration<double>(h->timeout_s);
    for (;;) {
        ncclResult_t state = ncclSuccess;
        const ncclResult_t r = n.api.ncclCommGetAsyncError(h->comm, &state);
        if (r != ncclSuccess) state = r;
        if (state == ncclSuccess) return PBRT_OK;
        if (state != ncclInProgress) {
            (void)n.api.ncclCommAbort(h->comm);
            h->aborted = true;
            return nccl_check(state, operation);
        }
        if (std::chrono::steady_clock::now() > deadline) {
            (void)n.api.ncclCommAbort(h->comm);
            h->aborted = true;
            return fail(PBRT_ERR_NCCL, std::string{operation} +
                                           " did not complete its enqueue in time; communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int after_call(comm_handle* h, ncclResult_t r, const char* operation) {
    if (r == ncclInProgress) return nccl_group_depth > 0 ? PBRT_OK : settle(h, operation);
    return nccl_check(r, operation);
}

}  // namespace

// =====================================================================
extern "C" {

const char* pbrt_last_error(void) { return tl_error.c_str(); }

int pbrt_available(void) {
    try {
        environment& env = env_raw();
        if (!env.cuda_ok || !env.nvrtc_ok) return 0;
        environment* e = nullptr;
        return ensure_init(e) == PBRT_OK ? 1 : 0;
    } catch (...) {
        return 0;
    }
}

int pbrt_init(void) {
    environment* env = nullptr;
    return ensure_init(env);
}

int pbrt_device_count(int* count) {
    if (count == nullptr) return fail(PBRT_ERR_INVALID, "count is null");
    environment* env = nullptr;
    int s = ensure_init(env);
    if (s != PBRT_OK) return s;
    *count = env->device_count;
    return PBRT_OK;
}

int pbrt_device_attribute(int device, int attribute, int* value) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuDeviceGetAttribute(
                     value, static_cast<CUdevice_attribute>(attribute),
                     env->devices[static_cast<size_t>(device)].device),
                 "cuDeviceGetAttribute");
}

int pbrt_device_name(int device, char* buffer, size_t length) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuDeviceGetName(buffer, static_cast<int>(length),
                                         env->devices[static_cast<size_t>(device)].device),
                 "cuDeviceGetName");
}

int pbrt_driver_version(int* version) {
    environment& env = env_raw();
    if (!env.cuda_ok) return fail(PBRT_ERR_UNAVAILABLE, "libcuda not found");
    return check(env, env.cu.cuDriverGetVersion(version), "cuDriverGetVersion");
}

int pbrt_nvrtc_version(int* major, int* minor) {
    environment& env = env_raw();
    if (!env.nvrtc_ok)
        return fail(PBRT_ERR_UNAVAILABLE, "CUDA JIT requires NVRTC at runtime");
    if (env.rtc.nvrtcVersion(major, minor) != NVRTC_SUCCESS)
        return fail(PBRT_ERR_UNAVAILABLE, "nvrtcVersion failed");
    return PBRT_OK;
}

// --------------------------------------------------------------- streams --
int pbrt_stream_current(int device, pbrt_stream* stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    auto& streams = tl_streams.streams;
    if (streams.size() <= static_cast<size_t>(device))
        streams.resize(static_cast<size_t>(device) + 1, nullptr);
    CUstream& st = streams[static_cast<size_t>(device)];
    if (st == nullptr) {
        s = check(*env, env->cu.cuStreamCreate(&st, CU_STREAM_NON_BLOCKING),
                  "cuStreamCreate");
        if (s != PBRT_OK) return s;
    }
    *stream = reinterpret_cast<pbrt_stream>(st);
    return PBRT_OK;
}

int pbrt_stream_create(int device, pbrt_stream* stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    CUstream st = nullptr;
    s = check(*env, env->cu.cuStreamCreate(&st, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
    *stream = reinterpret_cast<pbrt_stream>(st);
    return s;
}

int pbrt_stream_destroy(int device, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuStreamDestroy_v2(reinterpret_cast<CUstream>(stream)),
                 "cuStreamDestroy");
}

int pbrt_stream_synchronize(int device, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuStreamSynchronize(reinterpret_cast<CUstream>(stream)),
                 "cuStreamSynchronize");
}

int pbrt_event_create(int device, int enable_timing, pbrt_event* event) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    CUevent e = nullptr;
    s = check(*env,
              env->cu.cuEventCreate(&e, enable_timing ? CU_EVENT_DEFAULT
                                                      : CU_EVENT_DISABLE_TIMING),
              "cuEventCreate");
    *event = reinterpret_cast<pbrt_event>(e);
    return s;
}

int pbrt_event_destroy(int device, pbrt_event event) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuEventDestroy_v2(reinterpret_cast<CUevent>(event)),
                 "cuEventDestroy");
}

int pbrt_event_record(int device, pbrt_event event, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuEventRecord(reinterpret_cast<CUevent>(event),
                                       reinterpret_cast<CUstream>(stream)),
                 "cuEventRecord");
}

int pbrt_event_synchronize(int device, pbrt_event event) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuEventSynchronize(reinterpret_cast<CUevent>(event)),
                 "cuEventSynchronize");
}
int pbrt_event_query(int device, pbrt_event event, int* done) {
    if (event == nullptr || done == nullptr) return fail(PBRT_ERR_INVALID, "invalid event query");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    const CUresult r = env->cu.cuEventQuery(reinterpret_cast<CUevent>(event));
    if (r == CUDA_ERROR_NOT_READY) {
        *done = 0;
        return PBRT_OK;
    }
    *done = r == CUDA_SUCCESS ? 1 : 0;
    return check(*env, r, "cuEventQuery");
}


int pbrt_event_elapsed_ms(pbrt_event start, pbrt_event end, float* ms) {
    environment* env = nullptr;
    int s = ensure_init(env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuEventElapsedTime(ms, reinterpret_cast<CUevent>(start),
                                            reinterpret_cast<CUevent>(end)),
                 "cuEventElapsedTime");
}

int pbrt_stream_wait_event(int device, pbrt_stream stream, pbrt_event event) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuStreamWaitEvent(reinterpret_cast<CUstream>(stream),
                                           reinterpret_cast<CUevent>(event), 0),
                 "cuStreamWaitEvent");
}

// ---------------------------------------------------------------- memory --
int pbrt_mem_alloc_async(int device, size_t bytes, pbrt_stream stream,
                         uint64_t* pointer) {
    if (pointer == nullptr) return fail(PBRT_ERR_INVALID, "pointer is null");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (fault_fires(fault_alloc)) return PBRT_ERR_INJECTED;
    CUdeviceptr p = 0;
    s = check(*env, env->cu.cuMemAllocAsync(&p, bytes, reinterpret_cast<CUstream>(stream)),
              "cuMemAllocAsync");
    *pointer = static_cast<uint64_t>(p);
    return s;
}

int pbrt_mem_alloc(int device, size_t bytes, uint64_t* pointer) {
    if (pointer == nullptr) return fail(PBRT_ERR_INVALID, "pointer is null");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (fault_fires(fault_alloc)) return PBRT_ERR_INJECTED;
    CUdeviceptr p = 0;
    s = check(*env, env->cu.cuMemAlloc_v2(&p, bytes), "cuMemAlloc");
    *pointer = static_cast<uint64_t>(p);
    return s;
}

int pbrt_mem_free(int device, uint64_t pointer) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuMemFree_v2(static_cast<CUdeviceptr>(pointer)), "cuMemFree");
}

int pbrt_mem_free_async(int device, uint64_t pointer, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuMemFreeAsync(static_cast<CUdeviceptr>(pointer),
                                        reinterpret_cast<CUstream>(stream)),
                 "cuMemFreeAsync");
}

int pbrt_host_alloc(size_t bytes, void** pointer) {
    environment* env = nullptr;
    int s = use_device(0, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuMemHostAlloc(pointer, bytes, CU_MEMHOSTALLOC_PORTABLE),
                 "cuMemHostAlloc");
}

int pbrt_host_free(void* pointer) {
    environment* env = nullptr;
    int s = use_device(0, env);
    if (s != PBRT_OK) return s;
    return check(*env, env->cu.cuMemFreeHost(pointer), "cuMemFreeHost");
}

int pbrt_memcpy_h2d_async(int device, uint64_t dst, const void* src,
                          size_t bytes, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (fault_fires(fault_h2d)) return PBRT_ERR_INJECTED;
    if (bytes == 0) return PBRT_OK;
    return check(*env,
                 env->cu.cuMemcpyHtoDAsync_v2(static_cast<CUdeviceptr>(dst), src, bytes,
                                              reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyHtoDAsync");
}

int pbrt_memcpy_d2h_async(int device, void* dst, uint64_t src, size_t bytes,
                          pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (fault_fires(fault_d2h)) return PBRT_ERR_INJECTED;
    if (bytes == 0) return PBRT_OK;
    return check(*env,
                 env->cu.cuMemcpyDtoHAsync_v2(dst, static_cast<CUdeviceptr>(src), bytes,
                                              reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyDtoHAsync");
}

int pbrt_memcpy_d2d_async(int device, uint64_t dst, uint64_t src, size_t bytes,
                          pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (bytes == 0) return PBRT_OK;
    return check(*env,
                 env->cu.cuMemcpyDtoDAsync_v2(static_cast<CUdeviceptr>(dst),
                                              static_cast<CUdeviceptr>(src), bytes,
                                              reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyDtoDAsync");
}

int pbrt_memcpy_peer_async(int dst_device, uint64_t dst, int src_device,
                           uint64_t src, size_t bytes, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(src_device, env);
    if (s != PBRT_OK) return s;
    s = use_device(dst_device, env);
    if (s != PBRT_OK) return s;
    if (bytes == 0) return PBRT_OK;
    return check(*env,
                 env->cu.cuMemcpyPeerAsync(
                     static_cast<CUdeviceptr>(dst),
                     env->devices[static_cast<size_t>(dst_device)].context,
                     static_cast<CUdeviceptr>(src),
                     env->devices[static_cast<size_t>(src_device)].context, bytes,
                     reinterpret_cast<CUstream>(stream)),
                 "cuMemcpyPeerAsync");
}

int pbrt_memset_d32_async(int device, uint64_t dst, uint32_t value,
                          size_t count, pbrt_stream stream) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (count == 0) return PBRT_OK;
    return check(*env,
                 env->cu.cuMemsetD32Async(static_cast<CUdeviceptr>(dst), value, count,
                                          reinterpret_cast<CUstream>(stream)),
                 "cuMemsetD32Async");
}

int pbrt_enable_peer_access(int device, int peer) {
    environment* env = nullptr;
    int s = use_device(peer, env);
    if (s != PBRT_OK) return s;
    s = use_device(device, env);
    if (s != PBRT_OK) return s;
    int can = 0;
    s = check(*env,
              env->cu.cuDeviceCanAccessPeer(&can,
                                            env->devices[static_cast<size_t>(device)].device,
                                            env->devices[static_cast<size_t>(peer)].device),
              "cuDeviceCanAccessPeer");
    if (s != PBRT_OK) return s;
    if (!can) return fail(PBRT_ERR_UNAVAILABLE, "peer access not supported");
    CUresult r = env->cu.cuCtxEnablePeerAccess(
        env->devices[static_cast<size_t>(peer)].context, 0);
    if (r == CUDA_ERROR_PEER_ACCESS_ALREADY_ENABLED) return PBRT_OK;
    return check(*env, r, "cuCtxEnablePeerAccess");
}

// ------------------------------------------------------------------ JIT --
int pbrt_compile(const char* source, const char* const* options,
                 int option_count, int want_cubin, uint64_t* key) {
    if (source == nullptr || key == nullptr)
        return fail(PBRT_ERR_INVALID, "source or key is null");
    std::string text{source};
    text.push_back('\0');
    text.push_back(want_cubin ? 'C' : 'P');
    for (int i = 0; i < option_count; ++i) {
        text.push_back('\0');
        text += options[i];
    }
    const uint64_t h = finish_hash(hash_bytes(0xcbf29ce484222325ULL, text.data(), text.size()));
    module_cache& c = cache();
    {
        std::scoped_lock lock{c.mutex};
        auto it = c.images.find(h);
        if (it != c.images.end()) {
            if (it->second->text != text)
                return fail(PBRT_ERR_DRIVER,
                            "compile cache hash collision; refusing to reuse image");
            *key = h;
            return PBRT_OK;
        }
    }
    environment& env = env_raw();
    if (fault_fires(fault_compile)) return PBRT_ERR_INJECTED;

    // Optional on-disk cache.
    const std::string dir = disk_cache_dir();
    char name[32];
    std::snprintf(name, sizeof name, "%016llx", static_cast<unsigned long long>(h));
    if (!dir.empty()) {
        std::ifstream ktext(dir + "/" + name + ".key", std::ios::binary);
        std::ifstream kimg(dir + "/" + name + ".img", std::ios::binary);
        if (ktext && kimg) {
            std::string stored((std::istreambuf_iterator<char>(ktext)), {});
            if (stored == text) {
                auto img = std::make_unique<compiled_image>();
                img->text = text;
                img->image.assign((std::istreambuf_iterator<char>(kimg)), {});
                img->cubin = want_cubin != 0;
                g_disk_hits.fetch_add(1, std::memory_order_relaxed);
                std::scoped_lock lock{c.mutex};
                c.images.emplace(h, std::move(img));
                *key = h;
                return PBRT_OK;
            }
        }
    }

    if (!env.nvrtc_ok)
        return fail(PBRT_ERR_UNAVAILABLE, "CUDA JIT requires NVRTC at runtime");
    nvrtcProgram prog = nullptr;
    nvrtcResult r = env.rtc.nvrtcCreateProgram(&prog, source, "porch_kernel.cu", 0,
                                               nullptr, nullptr);
    if (r != NVRTC_SUCCESS)
        return fail(PBRT_ERR_COMPILE, std::string{"nvrtcCreateProgram failed: "} +
                                          env.rtc.nvrtcGetErrorString(r));
    struct guard {
        nvrtc_api* api;
        nvrtcProgram* p;
        ~guard() { (void)api->nvrtcDestroyProgram(p); }
    } g{&env.rtc, &prog};
    r = env.rtc.nvrtcCompileProgram(prog, option_count, options);
    if (r != NVRTC_SUCCESS) {
        size_t log_size = 0;
        std::string log;
        if (env.rtc.nvrtcGetProgramLogSize(prog, &log_size) == NVRTC_SUCCESS && log_size) {
            log.resize(log_size);
            (void)env.rtc.nvrtcGetProgramLog(prog, log.data());
            while (!log.empty() && log.back() == '\0') log.pop_back();
        }
        if (log.empty()) log = env.rtc.nvrtcGetErrorString(r);
        return fail(PBRT_ERR_COMPILE, log);
    }
    auto img = std::make_unique<compiled_image>();
    img->text = text;
    img->cubin = want_cubin != 0;
    size_t size = 0;
    if (want_cubin) {
        if (env.rtc.nvrtcGetCUBINSize(prog, &size) != NVRTC_SUCCESS || size == 0)
            return fail(PBRT_ERR_COMPILE,
                        "nvrtcGetCUBIN failed (was a real --gpu-architecture given?)");
        img->image.resize(size);
        if (env.rtc.nvrtcGetCUBIN(prog, img->image.data()) != NVRTC_SUCCESS)
            return fail(PBRT_ERR_COMPILE, "nvrtcGetCUBIN failed");
    } else {
        if (env.rtc.nvrtcGetPTXSize(prog, &size) != NVRTC_SUCCESS)
            return fail(PBRT_ERR_COMPILE, "nvrtcGetPTXSize failed");
        img->image.resize(size);
        if (env.rtc.nvrtcGetPTX(prog, img->image.data()) != NVRTC_SUCCESS)
            return fail(PBRT_ERR_COMPILE, "nvrtcGetPTX failed");
        if (img->image.empty() || img->image.back() != '\0') img->image.push_back('\0');
    }
    g_nvrtc_compiles.fetch_add(1, std::memory_order_relaxed);
    if (!dir.empty()) {
        // The image first, the key last: a key on disk implies its image.
        // A failed write only loses the cache entry.
        const std::string base = dir + "/" + name;
        if (write_file_atomically(base + ".img", img->image))
            (void)write_file_atomically(base + ".key", text);
    }
    std::scoped_lock lock{c.mutex};
    c.images.emplace(h, std::move(img));
    *key = h;
    return PBRT_OK;
}


int pbrt_compiled_image(uint64_t key, const void** image, size_t* size) {
    module_cache& c = cache();
    std::scoped_lock lock{c.mutex};
    auto it = c.images.find(key);
    if (it == c.images.end()) return fail(PBRT_ERR_INVALID, "unknown compiled image key");
    *image = it->second->image.data();
    *size = it->second->image.size();
    return PBRT_OK;
}

int pbrt_register_image(const void* image, size_t size, uint64_t* key) {
    if (image == nullptr || key == nullptr) return fail(PBRT_ERR_INVALID, "image or key is null");
    std::string bytes(static_cast<const char*>(image), size);
    std::string text = "\x01image\x01" + bytes;
    const uint64_t h = finish_hash(hash_bytes(0x84222325cbf29ce4ULL, text.data(), text.size()));
    module_cache& c = cache();
    std::scoped_lock lock{c.mutex};
    auto it = c.images.find(h);
    if (it == c.images.end()) {
        auto img = std::make_unique<compiled_image>();
        img->text = std::move(text);
        img->image = std::move(bytes);
        if (img->image.empty() || img->image.back() != '\0') img->image.push_back('\0');
        c.images.emplace(h, std::move(img));
    }
    *key = h;
    return PBRT_OK;
}

int pbrt_get_function(int device, uint64_t key, const char* name, pbrt_function* function) {
    if (name == nullptr || function == nullptr)
        return fail(PBRT_ERR_INVALID, "function name or output is null");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    module_cache& c = cache();
    std::scoped_lock lock{c.mutex};
    auto fkey = std::make_tuple(device, key, std::string{name});
    auto fit = c.functions.find(fkey);
    if (fit != c.functions.end()) {
        *function = reinterpret_cast<pbrt_function>(fit->second);
        return PBRT_OK;
    }
    auto mkey = std::make_pair(device, key);
    CUmodule module = nullptr;
    auto mit = c.modules.find(mkey);
    if (mit == c.modules.end()) {
        auto iit = c.images.find(key);
        if (iit == c.images.end()) return fail(PBRT_ERR_INVALID, "unknown compiled image key");
        s = check(*env, env->cu.cuModuleLoadData(&module, iit->second->image.data()),
                  "cuModuleLoadData");
        if (s != PBRT_OK) return s;
        c.modules.emplace(mkey, module);
    } else {
        module = mit->second;
    }
    CUfunction fn = nullptr;
    s = check(*env, env->cu.cuModuleGetFunction(&fn, module, name), "cuModuleGetFunction");
    if (s != PBRT_OK) return s;
    c.functions.emplace(fkey, fn);
    c.names.emplace(fn, std::string{name});
    *function = reinterpret_cast<pbrt_function>(fn);
    return PBRT_OK;
}

int pbrt_function_set_max_dynamic_smem(pbrt_function function, int bytes) {
    environment* env = nullptr;
    int s = ensure_init(env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuFuncSetAttribute(reinterpret_cast<CUfunction>(function),
                                            CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                            bytes),
                 "cuFuncSetAttribute");
}

int pbrt_function_attribute(pbrt_function function, int attribute, int* value) {
    environment* env = nullptr;
    int s = ensure_init(env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuFuncGetAttribute(value,
                                            static_cast<CUfunction_attribute>(attribute),
                                            reinterpret_cast<CUfunction>(function)),
                 "cuFuncGetAttribute");
}

int pbrt_occupancy(int device, pbrt_function function, int block_threads, size_t dynamic_smem,
                   int* blocks_per_sm) {
    if (function == nullptr || blocks_per_sm == nullptr || block_threads <= 0)
        return fail(PBRT_ERR_INVALID, "invalid occupancy query");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    return check(*env,
                 env->cu.cuOccupancyMaxActiveBlocksPerMultiprocessor(
                     blocks_per_sm, reinterpret_cast<CUfunction>(function), block_threads,
                     dynamic_smem),
                 "cuOccupancyMaxActiveBlocksPerMultiprocessor");
}

int pbrt_max_active_clusters(int device, pbrt_function function, int block_threads, size_t dynamic_smem,
                             unsigned cluster_x, int* clusters) {
    if (function == nullptr || clusters == nullptr || block_threads <= 0 || cluster_x == 0)
        return fail(PBRT_ERR_INVALID, "invalid cluster occupancy query");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    CUlaunchConfig config{};
    config.gridDimX = cluster_x;
    config.gridDimY = 1;
    config.gridDimZ = 1;
    config.blockDimX = static_cast<unsigned>(block_threads);
    config.blockDimY = 1;
    config.blockDimZ = 1;
    config.sharedMemBytes = static_cast<unsigned>(dynamic_smem);
    CUlaunchAttribute attribute{};
    attribute.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attribute.value.clusterDim.x = cluster_x;
    attribute.value.clusterDim.y = 1;
    attribute.value.clusterDim.z = 1;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return check(*env,
                 env->cu.cuOccupancyMaxActiveClusters(clusters, reinterpret_cast<CUfunction>(function), &config),
                 "cuOccupancyMaxActiveClusters");
}

int pbrt_launch(int device, pbrt_function function, const uint32_t* grid,
                const uint32_t* block, uint32_t dynamic_smem, pbrt_stream stream,
                void** params, const uint32_t* cluster) {
    return pbrt_launch_ex(device, function, grid, block, dynamic_smem, stream, params, cluster, 0u);
}

int pbrt_launch_ex(int device, pbrt_function function, const uint32_t* grid,
                   const uint32_t* block, uint32_t dynamic_smem, pbrt_stream stream,
                   void** params, const uint32_t* cluster, unsigned flags) {
    if (function == nullptr || grid == nullptr || block == nullptr)
        return fail(PBRT_ERR_INVALID, "launch function, grid or block is null");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    if (fault_fires(fault_launch)) return PBRT_ERR_INJECTED;
    CUlaunchConfig config{};
    config.gridDimX = grid[0];
    config.gridDimY = grid[1];
    config.gridDimZ = grid[2];
    config.blockDimX = block[0];
    config.blockDimY = block[1];
    config.blockDimZ = block[2];
    config.sharedMemBytes = dynamic_smem;
    config.hStream = reinterpret_cast<CUstream>(stream);
    CUlaunchAttribute attributes[2]{};
    unsigned n_attr = 0;
    if (cluster != nullptr && cluster[0] * cluster[1] * cluster[2] > 1) {
        attributes[n_attr].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
        attributes[n_attr].value.clusterDim.x = cluster[0];
        attributes[n_attr].value.clusterDim.y = cluster[1];
        attributes[n_attr].value.clusterDim.z = cluster[2];
        ++n_attr;
    }
    if ((flags & PBRT_LAUNCH_PDL) != 0) {
        attributes[n_attr].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attributes[n_attr].value.programmaticStreamSerializationAllowed = 1;
        ++n_attr;
    }
    if (n_attr > 0) {
        config.attrs = attributes;
        config.numAttrs = n_attr;
    }
    profiler& p = prof();
    const bool profiling = p.enabled;
    CUevent start = nullptr;
    CUevent stop = nullptr;
    if (profiling) {
        start = take_event(*env, device);
        stop = take_event(*env, device);
        if (start) (void)env->cu.cuEventRecord(start, config.hStream);
    }
    s = check(*env,
              env->cu.cuLaunchKernelEx(&config, reinterpret_cast<CUfunction>(function),
                                       params, nullptr),
              "cuLaunchKernel");
    if (s != PBRT_OK) return s;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (profiling && start && stop) {
        (void)env->cu.cuEventRecord(stop, config.hStream);
        std::scoped_lock lock{p.mutex};
        p.records.push_back({reinterpret_cast<CUfunction>(function), device, start, stop});
    }
    return PBRT_OK;
}

int pbrt_tensor_map_encode_tiled(void* out, int data_type, uint32_t rank,
                                 uint64_t global_address, const uint64_t* global_dims,
                                 const uint64_t* global_strides_bytes,
                                 const uint32_t* box_dims, const uint32_t* element_strides,
                                 int interleave, int swizzle, int l2_promotion,
                                 int oob_fill) {
    environment* env = nullptr;
    int s = ensure_init(env);
    if (s != PBRT_OK) return s;
    if (out == nullptr) return fail(PBRT_ERR_INVALID, "tensor map output is null");
    if ((global_address & 15u) != 0)
        return fail(PBRT_ERR_INVALID, "tensor map base address must be 16-byte aligned");
    for (uint32_t d = 0; d + 1 < rank; ++d) {
        if ((global_strides_bytes[d] & 15u) != 0)
            return fail(PBRT_ERR_INVALID, "tensor map strides must be multiples of 16 bytes");
    }
    return check(*env,
                 env->cu.cuTensorMapEncodeTiled(
                     static_cast<CUtensorMap*>(out),
                     static_cast<CUtensorMapDataType>(data_type), rank,
                     reinterpret_cast<void*>(global_address), global_dims,
                     global_strides_bytes, box_dims, element_strides,
                     static_cast<CUtensorMapInterleave>(interleave),
                     static_cast<CUtensorMapSwizzle>(swizzle),
                     static_cast<CUtensorMapL2promotion>(l2_promotion),
                     static_cast<CUtensorMapFloatOOBfill>(oob_fill)),
                 "cuTensorMapEncodeTiled");
}

// ------------------------------------------------------- error word --
int pbrt_error_word(int device, uint64_t* pointer) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    device_state& d = env->devices[static_cast<size_t>(device)];
    // A dedicated mutex: the helpers called below take device_mutex.
    static std::mutex* error_mutex = new std::mutex();
    std::scoped_lock lock{*error_mutex};
    if (d.error_block == 0) {
        pbrt_stream ps = nullptr;
        s = pbrt_stream_current(device, &ps);
        if (s != PBRT_OK) return s;
        CUstream st = reinterpret_cast<CUstream>(ps);
        CUdeviceptr p = 0;
        s = check(*env, env->cu.cuMemAlloc_v2(&p, 64), "cuMemAlloc");
        if (s != PBRT_OK) return s;
        s = check(*env, env->cu.cuMemsetD32Async(p, 0, 16, st), "cuMemsetD32Async");
        if (s != PBRT_OK) return s;
        s = check(*env, env->cu.cuStreamSynchronize(st), "cuStreamSynchronize");
        if (s != PBRT_OK) return s;
        d.error_block = p;
    }
    *pointer = static_cast<uint64_t>(d.error_block);
    return PBRT_OK;
}

int pbrt_error_check(int device, pbrt_stream stream, int* code) {
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    device_state& d = env->devices[static_cast<size_t>(device)];
    *code = 0;
    if (d.error_block == 0) return PBRT_OK;
    CUstream st = reinterpret_cast<CUstream>(stream);
    uint32_t words[16] = {};
    s = check(*env, env->cu.cuMemcpyDtoHAsync_v2(words, d.error_block, sizeof words, st),
              "cuMemcpyDtoHAsync");
    if (s != PBRT_OK) return s;
    s = check(*env, env->cu.cuStreamSynchronize(st), "cuStreamSynchronize");
    if (s != PBRT_OK) return s;
    if (words[0] != 0) {
        *code = static_cast<int>(words[0]);
        (void)env->cu.cuMemsetD32Async(d.error_block, 0, 16, st);
        (void)env->cu.cuStreamSynchronize(st);
        char msg[160];
        std::snprintf(msg, sizeof msg,
                      "device %d kernel error code %u (site %u, detail %u)", device,
                      words[0], words[1], words[2]);
        return fail(PBRT_ERR_DEVICE, msg);
    }
    return PBRT_OK;
}

// ---------------------------------------------------------- profiling --
int pbrt_profile_enable(int enable) {
    profiler& p = prof();
    std::scoped_lock lock{p.mutex};
    p.enabled = enable != 0;
    return PBRT_OK;
}

int pbrt_profile_read(char* buffer, size_t length) {
    environment* env = nullptr;
    int s = ensure_init(env);
    if (s != PBRT_OK) return s;
    profiler& p = prof();
    std::vector<launch_record> records;
    {
        std::scoped_lock lock{p.mutex};
        records.swap(p.records);
    }
    struct agg {
        uint64_t launches = 0;
        double ms = 0.0;
    };
    std::map<std::string, agg> totals;
    module_cache& c = cache();
    for (const launch_record& r : records) {
        (void)use_device(r.device, env);
        float ms = 0.0F;
        if (env->cu.cuEventSynchronize(r.stop) == CUDA_SUCCESS &&
            env->cu.cuEventElapsedTime(&ms, r.start, r.stop) == CUDA_SUCCESS) {
            std::string name;
            {
                std::scoped_lock lock{c.mutex};
                auto it = c.names.find(r.function);
                name = it == c.names.end() ? "?" : it->second;
            }
            agg& a = totals[name];
            a.launches += 1;
            a.ms += ms;
        }
        std::scoped_lock lock{p.mutex};
        p.free_events.emplace_back(r.device, r.start);
        p.free_events.emplace_back(r.device, r.stop);
    }
    std::string out;
    for (const auto& [name, a] : totals) {
        char line[512];
        std::snprintf(line, sizeof line, "%s\t%llu\t%.6f\n", name.c_str(),
                      static_cast<unsigned long long>(a.launches), a.ms);
        out += line;
    }
    if (buffer != nullptr && length > 0) {
        const size_t n = std::min(out.size(), length - 1);
        std::memcpy(buffer, out.data(), n);
        buffer[n] = '\0';
    }
    return PBRT_OK;
}

uint64_t pbrt_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

void pbrt_compile_stats(uint64_t* nvrtc_compiles, uint64_t* disk_cache_hits) {
    if (nvrtc_compiles) *nvrtc_compiles = g_nvrtc_compiles.load(std::memory_order_relaxed);
    if (disk_cache_hits) *disk_cache_hits = g_disk_hits.load(std::memory_order_relaxed);
}

int pbrt_fault_inject(const char* spec) { return parse_fault_spec(spec); }

// --------------------------------------------------------------- NCCL ----
int pbrt_nccl_available(void) { return nccl().ok ? 1 : 0; }

int pbrt_nccl_unique_id(char id[128]) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    ncclUniqueId uid{};
    int s = nccl_check(n.api.ncclGetUniqueId(&uid), "ncclGetUniqueId");
    if (s != PBRT_OK) return s;
    std::memcpy(id, uid.internal, sizeof uid.internal);
    return PBRT_OK;
}

int pbrt_nccl_init_all(int count, const int* devices, pbrt_comm* comms) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    if (count <= 0 || devices == nullptr || comms == nullptr)
        return fail(PBRT_ERR_INVALID, "invalid NCCL device list");
    if (fault_fires(fault_nccl_init)) return PBRT_ERR_INJECTED;
    environment* env = nullptr;
    for (int i = 0; i < count; ++i) {
        int s = use_device(devices[i], env);
        if (s != PBRT_OK) return s;
    }
    std::vector<ncclComm_t> raw(static_cast<size_t>(count), nullptr);
    int s = nccl_check(n.api.ncclCommInitAll(raw.data(), count, devices), "ncclCommInitAll");
    if (s != PBRT_OK) return s;
    for (int i = 0; i < count; ++i) {
        auto* h = new comm_handle{raw[static_cast<size_t>(i)], devices[i], false, 60.0};
        comms[i] = reinterpret_cast<pbrt_comm>(h);
    }
    return PBRT_OK;
}

int pbrt_nccl_init_rank(int nranks, const char id[128], int rank, int device,
                        double timeout_s, pbrt_comm* comm) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    if (fault_fires(fault_nccl_init)) return PBRT_ERR_INJECTED;
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    ncclUniqueId uid{};
    std::memcpy(uid.internal, id, sizeof uid.internal);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t raw = nullptr;
    ncclResult_t r = n.api.ncclCommInitRankConfig(&raw, nranks, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_check(r, "ncclCommInitRankConfig");
    const auto deadline = std::chrono::steady_clock::now() +
                          std::chrono::duration<double>(timeout_s);
    for (;;) {
        ncclResult_t state = ncclSuccess;
        r = n.api.ncclCommGetAsyncError(raw, &state);
        if (r != ncclSuccess) {
            (void)n.api.ncclCommAbort(raw);
            return nccl_check(r, "ncclCommGetAsyncError");
        }
        if (state == ncclSuccess) break;
        if (state != ncclInProgress) {
            (void)n.api.ncclCommAbort(raw);
            return nccl_check(state, "ncclCommInitRankConfig");
        }
        if (std::chrono::steady_clock::now() > deadline) {
            (void)n.api.ncclCommAbort(raw);
            return fail(PBRT_ERR_NCCL, "NCCL communicator init timed out");
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    *comm = reinterpret_cast<pbrt_comm>(new comm_handle{raw, device, false, timeout_s});
    return PBRT_OK;
}

int pbrt_nccl_group_start(void) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    const int s = nccl_check(n.api.ncclGroupStart(), "ncclGroupStart");
    if (s == PBRT_OK) ++nccl_group_depth;
    return s;
}

int pbrt_nccl_group_end(void) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    ncclResult_t r = n.api.ncclGroupEnd();
    if (nccl_group_depth > 0) --nccl_group_depth;
    if (r == ncclInProgress) return PBRT_OK;  // settled per communicator by pbrt_nccl_settle
    return nccl_check(r, "ncclGroupEnd");
}

int pbrt_nccl_settle(pbrt_comm comm) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr || h->aborted) return fail(PBRT_ERR_NCCL, "NCCL communicator is not usable");
    return settle(h, "NCCL group");
}

int pbrt_nccl_allgather_f32(pbrt_comm comm, uint64_t send, uint64_t recv,
                            size_t count_per_rank, pbrt_stream stream) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr || h->aborted) return fail(PBRT_ERR_NCCL, "NCCL communicator is not usable");
    if (fault_fires(fault_nccl_coll)) return PBRT_ERR_INJECTED;
    environment* env = nullptr;
    int s = use_device(h->device, env);
    if (s != PBRT_OK) return s;
    ncclResult_t r = n.api.ncclAllGather(reinterpret_cast<const void*>(send),
                                         reinterpret_cast<void*>(recv), count_per_rank,
                                         ncclFloat32, h->comm,
                                         reinterpret_cast<cudaStream_t>(stream));
    return after_call(h, r, "ncclAllGather");
}

int pbrt_nccl_send_f32(pbrt_comm comm, uint64_t send, size_t count, int peer,
                       pbrt_stream stream) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr || h->aborted) return fail(PBRT_ERR_NCCL, "NCCL communicator is not usable");
    if (fault_fires(fault_nccl_coll)) return PBRT_ERR_INJECTED;
    environment* env = nullptr;
    int s = use_device(h->device, env);
    if (s != PBRT_OK) return s;
    ncclResult_t r = n.api.ncclSend(reinterpret_cast<const void*>(send), count, ncclFloat32,
                                    peer, h->comm, reinterpret_cast<cudaStream_t>(stream));
    return after_call(h, r, "ncclSend");
}

int pbrt_nccl_recv_f32(pbrt_comm comm, uint64_t recv, size_t count, int peer,
                       pbrt_stream stream) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr || h->aborted) return fail(PBRT_ERR_NCCL, "NCCL communicator is not usable");
    if (fault_fires(fault_nccl_coll)) return PBRT_ERR_INJECTED;
    environment* env = nullptr;
    int s = use_device(h->device, env);
    if (s != PBRT_OK) return s;
    ncclResult_t r = n.api.ncclRecv(reinterpret_cast<void*>(recv), count, ncclFloat32, peer,
                                    h->comm, reinterpret_cast<cudaStream_t>(stream));
    return after_call(h, r, "ncclRecv");
}

int pbrt_nccl_wait(pbrt_comm comm, int device, pbrt_stream stream, double timeout_s) {
    nccl_env& n = nccl();
    if (!n.ok) return fail(PBRT_ERR_UNAVAILABLE, "libnccl.so.2 not found");
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr) return fail(PBRT_ERR_INVALID, "communicator is null");
    environment* env = nullptr;
    int s = use_device(device, env);
    if (s != PBRT_OK) return s;
    // Poll an event recorded behind the collective so the host never blocks
    // inside the driver on a peer that will not arrive.
    CUevent done = nullptr;
    s = check(*env, env->cu.cuEventCreate(&done, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
    if (s != PBRT_OK) return s;
    s = check(*env, env->cu.cuEventRecord(done, reinterpret_cast<CUstream>(stream)),
              "cuEventRecord");
    if (s != PBRT_OK) {
        (void)env->cu.cuEventDestroy_v2(done);
        return s;
    }
    const auto deadline = std::chrono::steady_clock::now() +
                          std::chrono::duration<double>(timeout_s);
    int status = PBRT_OK;
    for (;;) {
        ncclResult_t state = ncclSuccess;
        if (n.api.ncclCommGetAsyncError(h->comm, &state) == ncclSuccess &&
            state != ncclSuccess && state != ncclInProgress) {
            (void)n.api.ncclCommAbort(h->comm);
            h->aborted = true;
            status = nccl_check(state, "NCCL collective");
            break;
        }
        const CUresult q = env->cu.cuEventQuery(done);
        if (q == CUDA_SUCCESS) break;
        if (q != CUDA_ERROR_NOT_READY) {
            status = check(*env, q, "cuEventQuery");
            break;
        }
        if (std::chrono::steady_clock::now() > deadline) {
            (void)n.api.ncclCommAbort(h->comm);
            h->aborted = true;
            status = fail(PBRT_ERR_NCCL, "NCCL collective timed out; communicator aborted");
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    (void)env->cu.cuEventDestroy_v2(done);
    return status;
}

int pbrt_nccl_set_timeout(pbrt_comm comm, double timeout_s) {
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr) return fail(PBRT_ERR_INVALID, "communicator is null");
    if (!(timeout_s > 0.0)) return fail(PBRT_ERR_INVALID, "timeout must be positive");
    h->timeout_s = timeout_s;
    return PBRT_OK;
}

int pbrt_nccl_abort(pbrt_comm comm) {
    nccl_env& n = nccl();
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr) return PBRT_OK;
    if (!h->aborted && n.ok) (void)n.api.ncclCommAbort(h->comm);
    h->aborted = true;
    return PBRT_OK;
}

int pbrt_nccl_destroy(pbrt_comm comm) {
    nccl_env& n = nccl();
    auto* h = reinterpret_cast<comm_handle*>(comm);
    if (h == nullptr) return PBRT_OK;
    int s = PBRT_OK;
    if (!h->aborted && n.ok) {
        // Non-blocking communicators finalise first (flushing outstanding
        // work), bounded by the communicator's deadline, then are destroyed.
        ncclResult_t r = n.api.ncclCommFinalize(h->comm);
        s = r == ncclInProgress ? settle(h, "ncclCommFinalize") : nccl_check(r, "ncclCommFinalize");
        if (!h->aborted)
            s = s != PBRT_OK ? s : nccl_check(n.api.ncclCommDestroy(h->comm), "ncclCommDestroy");
    }
    delete h;
    return s;
}

}  // extern "C"
