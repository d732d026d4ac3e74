// libhawk_b200: the C ABI declared in include/hawk_b200.h.
//
// Artifacts are sm_100a CUBINs compiled by NVRTC from b200 units; they are
// loaded with the CUDA runtime's context-independent library API
// (cudaLibraryLoadData / cudaLibraryGetKernel / cudaLibraryGetGlobal) and
// launched with cudaLaunchKernel.  The CUDA runtime is linked statically, so
// the library loads (and reports its build facts) on a machine without a GPU
// driver; every device call then fails with HKB_ERR_CUDA and a message.
//
// The finish-tree kernels (hkb_cells_*) are compiled into this library.
#include "hawk_b200.h"

#include "hk/abi.cuh"
#include "hk/sample_sum.cuh"

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#ifndef HKB_BUILD_DIGEST
#define HKB_BUILD_DIGEST "unstamped"
#endif

namespace {

thread_local std::string g_error;

int fail(int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_error = buf;
    return status;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(HKB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

#define HKB_CUDA(call, what)                               \
    do {                                                   \
        cudaError_t hkb_err_ = (call);                     \
        if (hkb_err_ != cudaSuccess) return cuda_fail(hkb_err_, what); \
    } while (0)

enum class Kind { GRef, Handle, IntHandle, F64, F32, Int, NSamples };

bool kind_from_name(const char* name, Kind* out) {
    static const struct { const char* name; Kind kind; } table[] = {
        {"gref", Kind::GRef}, {"handle", Kind::Handle}, {"int_handle", Kind::IntHandle},
        {"f64", Kind::F64}, {"f32", Kind::F32}, {"int", Kind::Int}, {"nsamples", Kind::NSamples}};
    for (const auto& row : table)
        if (std::strcmp(row.name, name) == 0) {
            *out = row.kind;
            return true;
        }
    return false;
}

const uint64_t kLayout[5] = {sizeof(hk::abi::GRefMirror), sizeof(hk::abi::ScalarHandle),
                             sizeof(hk::abi::IntHandle), sizeof(hk::abi::index_t),
                             sizeof(hk::abi::PartitionTriple)};
const char* const kLayoutField[5] = {"GRefMirror", "ScalarHandle", "IntHandle", "index type",
                                     "PartitionTriple"};
const char kAbiTag[] = "aether-abi/2";

constexpr int kBlock = 256;   // every b200 entry is compiled __launch_bounds__(256)

// Sets `device` current for the scope, restoring the caller's on exit.
struct DeviceScope {
    int previous = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceScope(int device) {
        err = cudaGetDevice(&previous);
        if (err == cudaSuccess && previous != device) err = cudaSetDevice(device);
    }
    ~DeviceScope() {
        int now = -1;
        if (previous >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous) cudaSetDevice(previous);
    }
};

}  // namespace

struct hkb_library {
    cudaLibrary_t lib = nullptr;
    int device = 0;
    int sms = 0;
};

struct hkb_entry {
    hkb_library* lib = nullptr;
    cudaKernel_t kernel = nullptr;
    std::string name;
    int regs = 0;
    int blocks_per_sm = 0;
    int block = kBlock;          // threads per block this entry launches with
    unsigned dynamic_smem = 0;   // bytes per block the unit exports (hk_dynamic_smem_bytes)
    int team = 0;                // a team entry's threads (one block per lane), else 0
    bool spans_run = false;      // a team stage over keys, lane chunks or target cells
};

struct hkb_argblock {
    struct Cell {
        alignas(8) unsigned char bytes[40];
        Kind kind;
    };
    std::vector<Cell> cells;
    std::vector<void*> params;
};

extern "C" {

const char* hkb_last_error(void) { return g_error.c_str(); }

const char* hkb_build_digest(void) { return HKB_BUILD_DIGEST; }

int hkb_layout_sizes(uint64_t out[5]) {
    if (out == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_layout_sizes: null output");
    for (int k = 0; k < 5; ++k) out[k] = kLayout[k];
    return HKB_OK;
}

int hkb_device_count(int* count) {
    if (count == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_device_count: null output");
    *count = 0;
    const cudaError_t err = cudaGetDeviceCount(count);
    if (err != cudaSuccess) {
        *count = 0;
        cudaGetLastError();   // a machine without a driver: zero devices, not an error
    }
    return HKB_OK;
}

// ------------------------------------------------------------------ library

static int check_exports(hkb_library* lib) {
    void* dptr = nullptr;
    size_t bytes = 0;
    cudaError_t err = cudaLibraryGetGlobal(&dptr, &bytes, lib->lib, "eagle_abi_tag");
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(HKB_ERR_ABI, "the artifact exports no eagle_abi_tag: it is not a b200 unit");
    }
    char tag[64] = {0};
    if (bytes == 0 || bytes > sizeof tag)
        return fail(HKB_ERR_ABI, "the artifact's eagle_abi_tag has %zu bytes", bytes);
    HKB_CUDA(cudaMemcpy(tag, dptr, bytes, cudaMemcpyDeviceToHost), "reading eagle_abi_tag");
    if (std::strncmp(tag, kAbiTag, sizeof kAbiTag) != 0)
        return fail(HKB_ERR_ABI, "the artifact's eagle_abi_tag is '%s', this library packs '%s'", tag, kAbiTag);
    err = cudaLibraryGetGlobal(&dptr, &bytes, lib->lib, "eagle_layout_sizes");
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(HKB_ERR_ABI, "the artifact exports no eagle_layout_sizes");
    }
    if (bytes != sizeof kLayout)
        return fail(HKB_ERR_ABI, "the artifact's eagle_layout_sizes has %zu bytes, not %zu", bytes, sizeof kLayout);
    uint64_t sizes[5];
    HKB_CUDA(cudaMemcpy(sizes, dptr, bytes, cudaMemcpyDeviceToHost), "reading eagle_layout_sizes");
    for (int k = 0; k < 5; ++k)
        if (sizes[k] != kLayout[k])
            return fail(HKB_ERR_ABI, "layout mismatch in sizeof(%s): the artifact was built with %llu bytes, "
                        "this library packs %llu", kLayoutField[k], (unsigned long long)sizes[k],
                        (unsigned long long)kLayout[k]);
    return HKB_OK;
}

int hkb_library_load(const void* image, size_t size, int device, hkb_library** out) {
    if (image == nullptr || size == 0 || out == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_library_load: empty image or null output");
    *out = nullptr;
    DeviceScope scope(device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    auto* lib = new (std::nothrow) hkb_library();
    if (lib == nullptr) return fail(HKB_ERR_ARGUMENT, "out of host memory");
    lib->device = device;
    cudaError_t err = cudaLibraryLoadData(&lib->lib, image, nullptr, nullptr, 0, nullptr, nullptr, 0);
    if (err != cudaSuccess) {
        delete lib;
        return cuda_fail(err, "loading the sm_100a image");
    }
    err = cudaDeviceGetAttribute(&lib->sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) {
        cudaLibraryUnload(lib->lib);
        delete lib;
        return cuda_fail(err, "reading the SM count");
    }
    const int status = check_exports(lib);
    if (status != HKB_OK) {
        cudaLibraryUnload(lib->lib);
        delete lib;
        return status;
    }
    *out = lib;
    return HKB_OK;
}

int hkb_library_load_file(const char* path, int device, hkb_library** out) {
    if (path == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_library_load_file: null path");
    FILE* f = std::fopen(path, "rb");
    if (f == nullptr) return fail(HKB_ERR_NOT_FOUND, "cannot open artifact '%s'", path);
    std::vector<unsigned char> image;
    unsigned char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) image.insert(image.end(), buf, buf + n);
    std::fclose(f);
    return hkb_library_load(image.data(), image.size(), device, out);
}

void hkb_library_free(hkb_library* lib) {
    if (lib == nullptr) return;
    if (lib->lib != nullptr) cudaLibraryUnload(lib->lib);
    delete lib;
}

int hkb_library_errors(hkb_library* lib, unsigned* flags, int clear) {
    if (lib == nullptr || flags == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_library_errors: null argument");
    *flags = 0;
    DeviceScope scope(lib->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    void* dptr = nullptr;
    size_t bytes = 0;
    if (cudaLibraryGetGlobal(&dptr, &bytes, lib->lib, "hk_error_flags") != cudaSuccess || bytes != sizeof(unsigned)) {
        cudaGetLastError();
        return HKB_OK;
    }
    HKB_CUDA(cudaMemcpy(flags, dptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "reading hk_error_flags");
    if (clear) HKB_CUDA(cudaMemset(dptr, 0, sizeof(unsigned)), "clearing hk_error_flags");
    return HKB_OK;
}

int hkb_library_entry(hkb_library* lib, const char* name, hkb_entry** out) {
    if (lib == nullptr || name == nullptr || out == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_library_entry: null argument");
    *out = nullptr;
    DeviceScope scope(lib->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    cudaKernel_t kernel = nullptr;
    const cudaError_t err = cudaLibraryGetKernel(&kernel, lib->lib, name);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(HKB_ERR_NOT_FOUND, "the artifact has no entry '%s'", name);
    }
    auto* entry = new (std::nothrow) hkb_entry();
    if (entry == nullptr) return fail(HKB_ERR_ARGUMENT, "out of host memory");
    entry->lib = lib;
    entry->kernel = kernel;
    entry->name = name;
    cudaFuncAttributes attr;
    cudaError_t e2 = cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(kernel));
    if (e2 != cudaSuccess) {
        delete entry;
        return cuda_fail(e2, "reading the entry's attributes");
    }
    entry->regs = attr.numRegs;
    // A team entry (one block per lane) exports its threads per block,
    // hk_team_threads__<entry>; an entry of a unit with several entries its own
    // dynamic shared memory, hk_dynamic_smem_bytes__<entry>.
    const std::string team_sym = std::string("hk_team_threads__") + name;
    const std::string smem_sym = std::string("hk_dynamic_smem_bytes__") + name;
    void* tptr = nullptr;
    size_t tbytes = 0;
    if (cudaLibraryGetGlobal(&tptr, &tbytes, lib->lib, team_sym.c_str()) == cudaSuccess &&
        tbytes == sizeof(unsigned)) {
        unsigned threads = 0;
        e2 = cudaMemcpy(&threads, tptr, sizeof(unsigned), cudaMemcpyDeviceToHost);
        if (e2 != cudaSuccess) {
            delete entry;
            return cuda_fail(e2, "reading the team entry's threads");
        }
        if (threads == 0 || threads > 1024 || threads % 32 != 0) {
            delete entry;
            return fail(HKB_ERR_ABI, "entry '%s': a team of %u threads is not 1 to 32 whole warps", name, threads);
        }
        entry->team = static_cast<int>(threads);
        // A team stage over a block sum's keys, an ordered scatter's lane chunks
        // or its target cells exports hk_team_spans_run__<entry> = 1: its count
        // is those teams, which the run's sample count does not bound.
        const std::string spans_sym = std::string("hk_team_spans_run__") + name;
        void* gptr = nullptr;
        size_t gbytes = 0;
        if (cudaLibraryGetGlobal(&gptr, &gbytes, lib->lib, spans_sym.c_str()) == cudaSuccess &&
            gbytes == sizeof(unsigned)) {
            unsigned spans = 0;
            e2 = cudaMemcpy(&spans, gptr, sizeof(unsigned), cudaMemcpyDeviceToHost);
            if (e2 != cudaSuccess) {
                delete entry;
                return cuda_fail(e2, "reading the team stage's grid kind");
            }
            entry->spans_run = spans != 0;
        } else {
            cudaGetLastError();
        }
    } else {
        cudaGetLastError();
    }
    // A unit whose entry stages through dynamic shared memory exports its size.
    void* sptr = nullptr;
    size_t sbytes = 0;
    cudaError_t found = cudaLibraryGetGlobal(&sptr, &sbytes, lib->lib, smem_sym.c_str());
    if (found != cudaSuccess) {
        cudaGetLastError();
        found = cudaLibraryGetGlobal(&sptr, &sbytes, lib->lib, "hk_dynamic_smem_bytes");
    }
    if (found == cudaSuccess && sbytes == sizeof(unsigned)) {
        e2 = cudaMemcpy(&entry->dynamic_smem, sptr, sizeof(unsigned), cudaMemcpyDeviceToHost);
        if (e2 != cudaSuccess) {
            delete entry;
            return cuda_fail(e2, "reading the entry's shared-memory size");
        }
        e2 = cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(entry->dynamic_smem));
        if (e2 != cudaSuccess) {
            delete entry;
            return cuda_fail(e2, "raising the entry's shared-memory limit");
        }
    } else {
        cudaGetLastError();
    }
    // Threads per block: the size that keeps the most warps resident per SM (the
    // register file is the limit of a heavy entry: each quarter of the SM holds
    // 16384 registers, so at 98 registers a thread four warps fit a quarter and
    // at 96 five -- the unit asks for such a cap with __launch_bounds__(128, 5)),
    // the larger on a tie, never more than the entry was compiled for.  Every
    // frame indexes by blockDim; a staged entry's tiles assume 256 threads.
    const int candidates[] = {256, 128, 96, 64, 32};
    int best_warps = -1;
    for (int b : candidates) {
        if (entry->team != 0) b = entry->team;          // a team is its block
        else if (entry->dynamic_smem != 0 && b != kBlock) continue;
        else if (b > attr.maxThreadsPerBlock) continue;
        int bps = 0;
        e2 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, reinterpret_cast<const void*>(kernel), b,
                                                           entry->dynamic_smem);
        if (e2 != cudaSuccess) {
            delete entry;
            return cuda_fail(e2, "computing the entry's occupancy");
        }
        const int warps = bps * (b / 32);
        if (warps > best_warps) {
            best_warps = warps;
            entry->block = b;
            entry->blocks_per_sm = bps;
        }
        if (entry->team != 0) break;
    }
    if (entry->blocks_per_sm < 1) entry->blocks_per_sm = 1;
    *out = entry;
    return HKB_OK;
}

static int64_t grid_for(const hkb_entry* entry, int64_t count) {
    const int64_t cap = static_cast<int64_t>(entry->lib->sms) * entry->blocks_per_sm;
    // a team entry takes one lane per warp per trip; every other entry one
    // sample (or row) per thread
    const int64_t per_block = entry->team != 0 ? entry->block / 32 : entry->block;
    int64_t need = (count + per_block - 1) / per_block;
    if (need < 1) need = 1;
    return need < cap ? need : cap;
}

int hkb_entry_info(hkb_entry* entry, int* regs, int* blocks_per_sm, int* block, int64_t count,
                   int64_t* grid) {
    if (entry == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_entry_info: null entry");
    if (regs) *regs = entry->regs;
    if (blocks_per_sm) *blocks_per_sm = entry->blocks_per_sm;
    if (block) *block = entry->block;
    if (grid) *grid = grid_for(entry, count);
    return HKB_OK;
}

// ------------------------------------------------------------ argument block

int hkb_argblock_create(const char* const* kinds, size_t n, hkb_argblock** out) {
    if (out == nullptr || (n > 0 && kinds == nullptr))
        return fail(HKB_ERR_ARGUMENT, "hkb_argblock_create: null argument");
    *out = nullptr;
    auto* block = new (std::nothrow) hkb_argblock();
    if (block == nullptr) return fail(HKB_ERR_ARGUMENT, "out of host memory");
    block->cells.resize(n);
    block->params.resize(n, nullptr);
    for (size_t k = 0; k < n; ++k) {
        auto& cell = block->cells[k];
        if (kinds[k] == nullptr || !kind_from_name(kinds[k], &cell.kind)) {
            delete block;
            return fail(HKB_ERR_ARGUMENT, "slot %zu: unknown descriptor kind '%s'", k,
                        kinds[k] ? kinds[k] : "(null)");
        }
        std::memset(cell.bytes, 0, sizeof cell.bytes);
        // A fresh mirror is the POD's default: unit stride, a CUDA device.
        if (cell.kind == Kind::Handle || cell.kind == Kind::IntHandle) {
            auto* m = reinterpret_cast<hk::abi::ScalarHandle*>(cell.bytes);
            m->stride = 1;
            m->deviceType = 2;
        } else if (cell.kind == Kind::GRef) {
            auto* m = reinterpret_cast<hk::abi::GRefMirror*>(cell.bytes);
            m->sampleStride_ = 1;
            m->deviceType_ = 2;
        }
        block->params[k] = cell.bytes;
    }
    *out = block;
    return HKB_OK;
}

void hkb_argblock_free(hkb_argblock* block) { delete block; }

int hkb_argblock_bind(hkb_argblock* block, size_t slot, uintptr_t ptr, uint64_t samples,
                      uint64_t stride, int32_t device_type, int32_t device_id) {
    if (block == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_argblock_bind: null block");
    if (slot >= block->cells.size())
        return fail(HKB_ERR_ARGUMENT, "slot %zu is outside this block's %zu slots", slot, block->cells.size());
    auto& cell = block->cells[slot];
    switch (cell.kind) {
        case Kind::GRef: {
            auto* m = reinterpret_cast<hk::abi::GRefMirror*>(cell.bytes);
            m->data_ = reinterpret_cast<double*>(ptr);
            m->samples_ = samples;
            m->compStride_ = samples * stride;
            m->sampleStride_ = stride;
            m->deviceType_ = device_type;
            m->deviceId_ = device_id;
            return HKB_OK;
        }
        case Kind::Handle:
        case Kind::IntHandle: {
            auto* m = reinterpret_cast<hk::abi::ScalarHandle*>(cell.bytes);
            m->data = reinterpret_cast<void*>(ptr);
            m->samples = samples;
            m->stride = stride;
            m->deviceType = device_type;
            m->deviceId = device_id;
            return HKB_OK;
        }
        default:
            break;
    }
    // A by-value slot copies the value at `ptr` (a caller's temporary).
    if (ptr == 0)
        return fail(HKB_ERR_ARGUMENT, "slot %zu is a by-value slot and needs the address of its value", slot);
    const void* src = reinterpret_cast<const void*>(ptr);
    switch (cell.kind) {
        case Kind::F64: std::memcpy(cell.bytes, src, sizeof(double)); break;
        case Kind::F32: std::memcpy(cell.bytes, src, sizeof(float)); break;
        case Kind::Int: std::memcpy(cell.bytes, src, sizeof(long long)); break;
        case Kind::NSamples: std::memcpy(cell.bytes, src, sizeof(hk::abi::index_t)); break;
        default: break;
    }
    return HKB_OK;
}

int hkb_argblock_rebind(hkb_argblock* block, const int64_t* slots, const int64_t* ptrs, size_t n) {
    if (block == nullptr || (n > 0 && (slots == nullptr || ptrs == nullptr)))
        return fail(HKB_ERR_ARGUMENT, "hkb_argblock_rebind: null argument");
    for (size_t i = 0; i < n; ++i) {
        const int64_t s = slots[i];
        if (s < 0 || static_cast<size_t>(s) >= block->cells.size())
            return fail(HKB_ERR_ARGUMENT, "rebind: slot %lld is outside this block's %zu slots",
                        (long long)s, block->cells.size());
        auto& cell = block->cells[static_cast<size_t>(s)];
        if (cell.kind == Kind::GRef) {
            reinterpret_cast<hk::abi::GRefMirror*>(cell.bytes)->data_ = reinterpret_cast<double*>(ptrs[i]);
        } else if (cell.kind == Kind::Handle || cell.kind == Kind::IntHandle) {
            reinterpret_cast<hk::abi::ScalarHandle*>(cell.bytes)->data = reinterpret_cast<void*>(ptrs[i]);
        } else {
            return fail(HKB_ERR_ARGUMENT, "rebind: slot %lld is a by-value slot and carries no pointer; "
                        "set it with bind (rebind is the pointer path)", (long long)s);
        }
    }
    return HKB_OK;
}

// --------------------------------------------------------------------- launch

int hkb_entry_launch(hkb_entry* entry, hkb_argblock* block, int64_t base, int64_t count,
                     int64_t n_samples, void* stream) {
    if (entry == nullptr || block == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_entry_launch: null argument");
    if (entry->spans_run) {
        if (base != 0 || count < 0 || n_samples < 0)
            return fail(HKB_ERR_RANGE, "team stage '%s' spans the run: base must be 0 and count its teams, "
                        "got base %lld, count %lld", entry->name.c_str(), (long long)base, (long long)count);
    } else if (base < 0 || count < 0 || base + count > n_samples) {
        return fail(HKB_ERR_RANGE, "partition [%lld, %lld) is outside the %lld samples",
                    (long long)base, (long long)(base + count), (long long)n_samples);
    }
    if (count == 0) return HKB_OK;
    DeviceScope scope(entry->lib->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    std::vector<void*> args(block->params);
    long long b = base, c = count, ns = n_samples;
    args.push_back(&b);
    args.push_back(&c);
    args.push_back(&ns);
    // A launch of fewer samples than one block per SM (a reader stage of a few
    // thousand lanes, a small partition) runs in smaller blocks, so that every
    // SM takes a share: whole warps, at least 32 threads.  Entries that stage
    // through shared memory keep their block.
    int threads = entry->block;
    if (entry->team == 0 && entry->dynamic_smem == 0 && count < static_cast<int64_t>(entry->lib->sms) * threads) {
        const int64_t per_sm = (count + entry->lib->sms - 1) / entry->lib->sms;
        const int64_t warps = (per_sm + 31) / 32;
        threads = static_cast<int>(warps < 1 ? 32 : (warps * 32 < threads ? warps * 32 : threads));
    }
    const int64_t per_block = entry->team != 0 ? threads / 32 : threads;
    const int64_t need = (count + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(entry->lib->sms) * entry->blocks_per_sm * (entry->block / threads);
    const dim3 grid(static_cast<unsigned>(need < 1 ? 1 : (need < cap ? need : cap)));
    const cudaError_t err = cudaLaunchKernel(reinterpret_cast<const void*>(entry->kernel), grid, dim3(threads),
                                             args.data(), entry->dynamic_smem, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "launching the entry");
    return HKB_OK;
}

int hkb_entry_launch_persist(hkb_entry* entry, hkb_argblock* block, int64_t base, int64_t count,
                             int64_t n_samples, uint32_t* next, uint64_t* util, uint32_t* steps,
                             uint64_t* stepsum, uint32_t chunk, int64_t grid, void* stream) {
    if (entry == nullptr || block == nullptr || next == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_entry_launch_persist: null entry, block or claim counter");
    if (base < 0 || count < 0 || base + count > n_samples)
        return fail(HKB_ERR_RANGE, "partition [%lld, %lld) is outside the %lld samples",
                    (long long)base, (long long)(base + count), (long long)n_samples);
    if (count >= (int64_t(1) << 31))
        return fail(HKB_ERR_RANGE, "a persistent launch claims samples with a 32-bit counter: %lld samples "
                    "is 2^31 or more; split the range", (long long)count);
    if (grid < 0) return fail(HKB_ERR_ARGUMENT, "hkb_entry_launch_persist: negative grid %lld", (long long)grid);
    if (count == 0) return HKB_OK;
    DeviceScope scope(entry->lib->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    std::vector<void*> args(block->params);
    long long b = base, c = count, ns = n_samples;
    unsigned ch = chunk;
    args.push_back(&b);
    args.push_back(&c);
    args.push_back(&ns);
    args.push_back(&next);
    args.push_back(&util);
    args.push_back(&steps);
    args.push_back(&stepsum);
    args.push_back(&ch);
    // a resident grid: every claim loop runs until the counter passes count
    const int64_t g = grid > 0 ? grid : grid_for(entry, count);
    const cudaError_t err = cudaLaunchKernel(reinterpret_cast<const void*>(entry->kernel),
                                             dim3(static_cast<unsigned>(g)), dim3(entry->block), args.data(),
                                             entry->dynamic_smem, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "launching the persistent entry");
    return HKB_OK;
}

int hkb_entry_launch_range(hkb_entry* entry, hkb_argblock* block, int64_t base, int64_t count,
                           int64_t n_samples, uint32_t* steps, uint64_t* stepsum, void* stream) {
    if (entry == nullptr || block == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_entry_launch_range: null argument");
    if (base < 0 || count < 0 || base + count > n_samples)
        return fail(HKB_ERR_RANGE, "partition [%lld, %lld) is outside the %lld samples",
                    (long long)base, (long long)(base + count), (long long)n_samples);
    if (count == 0) return HKB_OK;
    DeviceScope scope(entry->lib->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    std::vector<void*> args(block->params);
    long long b = base, c = count, ns = n_samples;
    args.push_back(&b);
    args.push_back(&c);
    args.push_back(&ns);
    args.push_back(&steps);
    args.push_back(&stepsum);
    // the lane frame's grid: every resident slot, capped by the samples (whole
    // warps always: the per-warp report after the frame needs all 32 lanes)
    const int64_t threads = entry->block;
    const int64_t need = (count + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(entry->lib->sms) * entry->blocks_per_sm;
    const dim3 grid(static_cast<unsigned>(need < 1 ? 1 : (need < cap ? need : cap)));
    const cudaError_t err = cudaLaunchKernel(reinterpret_cast<const void*>(entry->kernel), grid,
                                             dim3(static_cast<unsigned>(threads)), args.data(), entry->dynamic_smem,
                                             static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "launching the range entry");
    return HKB_OK;
}

}  // extern "C"

// ------------------------------------------------------------ the finish tree

namespace {

constexpr int kMaxCols = 8;

struct Columns {
    const void* hi[kMaxCols];
    const void* comp[kMaxCols];
};

// One block per (leaf, column): the slot walk (16 terms per slot, Neumaier
// steps in order), then the halving tree over the 256 slots
// (hawk/_cells.py:71-91).
template <class T, int OP>
__global__ void __launch_bounds__(hk::ss::kSlots) leaves_kernel(Columns cols, long long rows, long long leaves,
                                                                  T* leaf_hi, T* leaf_comp) {
    __shared__ T sh[hk::ss::kSlots];
    __shared__ T sc[hk::ss::kSlots];
    const int col = blockIdx.y;
    const long long leaf = blockIdx.x;
    const T* hi = static_cast<const T*>(cols.hi[col]);
    const T* comp = static_cast<const T*>(cols.comp[col]);
    const long long r0 = leaf * hk::ss::kLeaf;
    const long long left = rows - r0;
    const int cnt = static_cast<int>(left < hk::ss::kLeaf ? left : hk::ss::kLeaf);
    const int live = cnt < hk::ss::kSlots ? cnt : hk::ss::kSlots;
    const int s = threadIdx.x;
    T h = T(0), c = T(0);
    if (cnt == hk::ss::kLeaf) {
        // A full leaf: all 16 terms of the slot (and their compensations) are
        // loaded before the first step, so the loads are in flight together.
        T xh[hk::ss::kTerms], xc[hk::ss::kTerms];
#pragma unroll
        for (int k = 0; k < hk::ss::kTerms; ++k) {
            xh[k] = hi[r0 + k * hk::ss::kSlots + s];
            xc[k] = (OP == hk::ss::kSum && comp != nullptr) ? comp[r0 + k * hk::ss::kSlots + s] : T(0);
        }
        h = xh[0];
        c = hk::ss::finite(h) ? xc[0] : T(0);
#pragma unroll
        for (int k = 1; k < hk::ss::kTerms; ++k) hk::ss::neumaier_add<OP>(h, c, xh[k], xc[k]);
    } else if (s < live) {
        h = hi[r0 + s];
        c = (OP == hk::ss::kSum && comp != nullptr) ? comp[r0 + s] : T(0);
        if (!hk::ss::finite(h)) c = T(0);
#pragma unroll 1
        for (int k = 1; k < hk::ss::kTerms; ++k) {
            const int rest = cnt - k * hk::ss::kSlots;
            const int m = rest < live ? rest : live;
            if (m <= 0) break;
            if (s < m) {
                const long long r = r0 + static_cast<long long>(k) * hk::ss::kSlots + s;
                const T xc = (OP == hk::ss::kSum && comp != nullptr) ? comp[r] : T(0);
                hk::ss::neumaier_add<OP>(h, c, hi[r], xc);
            }
        }
    }
    sh[s] = h;
    sc[s] = c;
    __syncthreads();
#pragma unroll 1
    for (int off = hk::ss::kSlots / 2; off > 0; off >>= 1) {
        const int lim = live > off ? (off < live - off ? off : live - off) : 0;
        T a = T(0), ac = T(0);
        if (s < lim) {
            a = sh[s];
            ac = sc[s];
            hk::ss::tree_join<OP>(a, ac, sh[s + off], sc[s + off]);
        }
        __syncthreads();
        if (s < lim) {
            sh[s] = a;
            sc[s] = ac;
        }
        __syncthreads();
    }
    if (s == 0) {
        leaf_hi[col * leaves + leaf] = sh[0];
        leaf_comp[col * leaves + leaf] = sc[0];
    }
}

// One block per column: the pairwise levels over the leaves, in place (the
// partial of level s sits at index k * 2^s), then hi + comp (hawk/_cells.py:108-119).
// Leaf j of column k is at [k * col_stride + j * elem_stride].  With out_comp
// the root's (hi, comp) pair is written instead of hi + comp: the root of an
// aligned subtree, which a later tree joins with the others.
template <class T, int OP>
__global__ void __launch_bounds__(1024) tree_kernel(T* leaf_hi, T* leaf_comp, long long leaves, long long elem_stride,
                                                   long long col_stride, T* out, T* out_comp) {
    const int col = blockIdx.x;
    T* h = leaf_hi + col * col_stride;
    T* c = leaf_comp + col * col_stride;
    for (long long st = 1; st < leaves; st <<= 1) {
        for (long long idx = static_cast<long long>(threadIdx.x) * 2 * st; idx < leaves;
             idx += static_cast<long long>(blockDim.x) * 2 * st) {
            if (idx + st < leaves) {
                T a = h[idx * elem_stride], ac = c[idx * elem_stride];
                hk::ss::tree_join<OP>(a, ac, h[(idx + st) * elem_stride], c[(idx + st) * elem_stride]);
                h[idx * elem_stride] = a;
                c[idx * elem_stride] = ac;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const T v = h[0];
        if (out_comp != nullptr) {
            out[col] = v;
            out_comp[col] = c[0];
        } else {
            out[col] = (OP == hk::ss::kSum) ? (hk::ss::finite(v) ? v + c[0] : v) : v;
        }
    }
}

template <class T>
int launch_leaves(int op, const Columns& cols, int ncols, int64_t rows, int64_t leaves, void* lh, void* lc,
                  cudaStream_t stream) {
    const dim3 grid(static_cast<unsigned>(leaves), static_cast<unsigned>(ncols));
    T* h = static_cast<T*>(lh);
    T* c = static_cast<T*>(lc);
    switch (op) {
        case HKB_OP_SUM: leaves_kernel<T, hk::ss::kSum><<<grid, hk::ss::kSlots, 0, stream>>>(cols, rows, leaves, h, c); break;
        case HKB_OP_MAX: leaves_kernel<T, hk::ss::kMax><<<grid, hk::ss::kSlots, 0, stream>>>(cols, rows, leaves, h, c); break;
        default: leaves_kernel<T, hk::ss::kMin><<<grid, hk::ss::kSlots, 0, stream>>>(cols, rows, leaves, h, c); break;
    }
    HKB_CUDA(cudaGetLastError(), "launching the leaf stage");
    return HKB_OK;
}

template <class T>
int launch_tree(int op, int ncols, void* lh, void* lc, int64_t leaves, int64_t elem_stride, int64_t col_stride,
                void* out, void* out_comp, cudaStream_t stream) {
    T* h = static_cast<T*>(lh);
    T* c = static_cast<T*>(lc);
    T* o = static_cast<T*>(out);
    T* oc = static_cast<T*>(out_comp);
    const int threads = 1024;
    switch (op) {
        case HKB_OP_SUM:
            tree_kernel<T, hk::ss::kSum><<<ncols, threads, 0, stream>>>(h, c, leaves, elem_stride, col_stride, o, oc);
            break;
        case HKB_OP_MAX:
            tree_kernel<T, hk::ss::kMax><<<ncols, threads, 0, stream>>>(h, c, leaves, elem_stride, col_stride, o, oc);
            break;
        default:
            tree_kernel<T, hk::ss::kMin><<<ncols, threads, 0, stream>>>(h, c, leaves, elem_stride, col_stride, o, oc);
            break;
    }
    HKB_CUDA(cudaGetLastError(), "launching the tree stage");
    return HKB_OK;
}

int check_cells(int op, int dtype, int ncols) {
    if (op != HKB_OP_SUM && op != HKB_OP_MAX && op != HKB_OP_MIN) return fail(HKB_ERR_ARGUMENT, "unknown op %d", op);
    if (dtype != HKB_F64 && dtype != HKB_F32) return fail(HKB_ERR_ARGUMENT, "unknown dtype %d", dtype);
    if (ncols < 1 || ncols > kMaxCols) return fail(HKB_ERR_RANGE, "ncols %d is outside 1..%d", ncols, kMaxCols);
    return HKB_OK;
}

int64_t leaves_of(int64_t rows) { return (rows + HKB_LEAF_ROWS - 1) / HKB_LEAF_ROWS; }

}  // namespace

extern "C" {

int hkb_cells_leaves(int op, int dtype, int ncols, const void* const* hi, const void* const* comp,
                     int64_t rows, void* leaf_hi, void* leaf_comp, void* stream) {
    int status = check_cells(op, dtype, ncols);
    if (status != HKB_OK) return status;
    if (rows < 1) return fail(HKB_ERR_RANGE, "a finish needs at least one row, got %lld", (long long)rows);
    if (hi == nullptr || leaf_hi == nullptr || leaf_comp == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_cells_leaves: null pointer");
    const int64_t leaves = leaves_of(rows);
    if (leaves > 2147483647LL) return fail(HKB_ERR_RANGE, "too many leaves (%lld)", (long long)leaves);
    Columns cols;
    for (int k = 0; k < kMaxCols; ++k) {
        cols.hi[k] = k < ncols ? hi[k] : nullptr;
        cols.comp[k] = (k < ncols && comp != nullptr) ? comp[k] : nullptr;
        if (k < ncols && cols.hi[k] == nullptr) return fail(HKB_ERR_ARGUMENT, "column %d has no rows", k);
        if (k < ncols && op == HKB_OP_SUM && cols.comp[k] == nullptr)
            return fail(HKB_ERR_ARGUMENT, "column %d of a sum has no compensation rows", k);
    }
    auto s = static_cast<cudaStream_t>(stream);
    return dtype == HKB_F64 ? launch_leaves<double>(op, cols, ncols, rows, leaves, leaf_hi, leaf_comp, s)
                            : launch_leaves<float>(op, cols, ncols, rows, leaves, leaf_hi, leaf_comp, s);
}

int hkb_cells_tree(int op, int dtype, int ncols, void* leaf_hi, void* leaf_comp, int64_t leaves, void* out,
                   void* stream) {
    int status = check_cells(op, dtype, ncols);
    if (status != HKB_OK) return status;
    if (leaves < 1) return fail(HKB_ERR_RANGE, "a tree needs at least one leaf");
    if (leaf_hi == nullptr || leaf_comp == nullptr || out == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_cells_tree: null pointer");
    auto s = static_cast<cudaStream_t>(stream);
    return dtype == HKB_F64 ? launch_tree<double>(op, ncols, leaf_hi, leaf_comp, leaves, 1, leaves, out, nullptr, s)
                            : launch_tree<float>(op, ncols, leaf_hi, leaf_comp, leaves, 1, leaves, out, nullptr, s);
}

int hkb_cells_tree_ex(int op, int dtype, int ncols, void* hi, void* comp, int64_t count, int64_t elem_stride,
                      int64_t col_stride, void* out, void* out_comp, void* stream) {
    int status = check_cells(op, dtype, ncols);
    if (status != HKB_OK) return status;
    if (count < 1) return fail(HKB_ERR_RANGE, "a tree needs at least one leaf");
    if (elem_stride < 1 || col_stride < 0)
        return fail(HKB_ERR_RANGE, "strides %lld, %lld: the element stride is positive", (long long)elem_stride,
                    (long long)col_stride);
    if (hi == nullptr || comp == nullptr || out == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_cells_tree_ex: null pointer");
    auto s = static_cast<cudaStream_t>(stream);
    return dtype == HKB_F64
               ? launch_tree<double>(op, ncols, hi, comp, count, elem_stride, col_stride, out, out_comp, s)
               : launch_tree<float>(op, ncols, hi, comp, count, elem_stride, col_stride, out, out_comp, s);
}

size_t hkb_cells_scratch_bytes(int dtype, int ncols, int64_t rows) {
    const size_t elem = dtype == HKB_F32 ? sizeof(float) : sizeof(double);
    const int64_t leaves = rows < 1 ? 1 : leaves_of(rows);
    return 2 * static_cast<size_t>(ncols < 1 ? 1 : ncols) * static_cast<size_t>(leaves) * elem;
}

int hkb_cells_finish(int op, int dtype, int ncols, const void* const* hi, const void* const* comp,
                     int64_t rows, void* scratch, void* out, void* stream) {
    if (scratch == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_cells_finish: null scratch");
    const size_t elem = dtype == HKB_F32 ? sizeof(float) : sizeof(double);
    const int64_t leaves = leaves_of(rows < 1 ? 1 : rows);
    char* lh = static_cast<char*>(scratch);
    char* lc = lh + static_cast<size_t>(ncols < 1 ? 1 : ncols) * static_cast<size_t>(leaves) * elem;
    int status = hkb_cells_leaves(op, dtype, ncols, hi, comp, rows, lh, lc, stream);
    if (status != HKB_OK) return status;
    return hkb_cells_tree(op, dtype, ncols, lh, lc, leaves, out, stream);
}

}  // extern "C"

// ------------------------------------------------ the allocation-free finish
//
// hkb_cells_finish needs its caller to hand it scratch for the leaf partials.
// Some callers have no way to get device memory at the point they finish a
// reduction: a host framework that owns every device allocation and hands its
// plugins only their inputs and outputs, or a real-time loop whose memory
// budget is fixed before it starts and which must never enter the CUDA
// allocator.  For them, hkb_cells_finish_noalloc keeps the leaf partials in
// the array below, which lives in this library's device image: every GPU that
// loads the library holds it (HKB_NOALLOC_LEAF_CAP partials of hi and comp,
// 128 KiB) until the process exits, and nothing is allocated per call.

namespace {

static __device__ __align__(256) double g_noalloc_leaves[2 * HKB_NOALLOC_LEAF_CAP];

constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// The device address of g_noalloc_leaves on the current device, resolved once
// per device (host code cannot use the symbol itself as an address).
int noalloc_scratch(void** out) {
    int device = -1;
    HKB_CUDA(cudaGetDevice(&device), "reading the current device");
    if (device < 0 || device >= kMaxDevices)
        return fail(HKB_ERR_RANGE, "device %d is beyond the %d devices the static scratch table covers",
                    device, kMaxDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[device] == nullptr) {
        void* p = nullptr;
        HKB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_leaves), "resolving the static leaf scratch");
        g_noalloc_ptr[device] = p;
    }
    *out = g_noalloc_ptr[device];
    return HKB_OK;
}

}  // namespace

extern "C" int hkb_cells_finish_noalloc(int op, int dtype, int ncols, const void* const* hi,
                                         const void* const* comp, int64_t rows, void* out, void* stream) {
    int status = check_cells(op, dtype, ncols);
    if (status != HKB_OK) return status;
    if (rows < 1) return fail(HKB_ERR_RANGE, "a finish needs at least one row, got %lld", (long long)rows);
    const int64_t leaves = leaves_of(rows);
    if (leaves * ncols > HKB_NOALLOC_LEAF_CAP)
        return fail(HKB_ERR_RANGE,
                    "%d columns of %lld rows need %lld leaf partials, more than the %d the static scratch "
                    "holds (at most %lld rows per column at this column count); use hkb_cells_finish with "
                    "caller scratch", ncols, (long long)rows, (long long)(leaves * ncols), HKB_NOALLOC_LEAF_CAP,
                    (long long)(HKB_NOALLOC_LEAF_CAP / ncols) * HKB_LEAF_ROWS);
    void* scratch = nullptr;
    status = noalloc_scratch(&scratch);
    if (status != HKB_OK) return status;
    // Every partial the tree stage reads is written by the leaf stage of the
    // same call first, so nothing in the scratch has to start at zero.
    const size_t elem = dtype == HKB_F32 ? sizeof(float) : sizeof(double);
    char* lh = static_cast<char*>(scratch);
    char* lc = lh + static_cast<size_t>(HKB_NOALLOC_LEAF_CAP) * elem;
    status = hkb_cells_leaves(op, dtype, ncols, hi, comp, rows, lh, lc, stream);
    if (status != HKB_OK) return status;
    return hkb_cells_tree(op, dtype, ncols, lh, lc, leaves, out, stream);
}

// ------------------------------------------- cells across GPUs, peer memory
//
// The last step of a sharded finish without a collective library: every rank
// folds its leaves to one (hi, comp) root per column and stores the root into
// every rank's exchange area over NVLink (plain peer stores through CUDA IPC
// mappings), each 32-bit half of a value in its own 8-byte word beside the
// round's tag -- a word is written and read whole, so a reader that sees the
// round's tag in a word has that word's half, and no fence or flag is needed
// (the low-latency form collective libraries use for small messages).  Each
// rank waits (bounded) until every rank's words of the round carry the tag in
// its own area, and folds the roots in rank order.  The area keeps two round
// parities, so a rank one round ahead writes the other parity's words and never
// overwrites a root its peer is still to read: a rank can only start round
// s + 2 after every rank has published round s + 1, which each does only after
// its round s finished.

namespace {

constexpr int kPeerRanks = HKB_PEER_MAX_RANKS;
constexpr int kPeerWords = 4;                                   // hi's two halves, then comp's
constexpr size_t kPeerWordsAt = 256;                            // after the status word
constexpr size_t kPeerAreaBytes = kPeerWordsAt + 2 * kPeerRanks * kMaxCols * kPeerWords * 8 + 256;
constexpr unsigned long long kPeerWaitNs = 2000000000ull;

struct PeerAreas {
    unsigned char* area[kPeerRanks];
};

__device__ __forceinline__ unsigned long long peer_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long* peer_words(unsigned char* area, int parity, int rank, int col) {
    return reinterpret_cast<unsigned long long*>(area + kPeerWordsAt) +
           ((parity * kPeerRanks + rank) * kMaxCols + col) * kPeerWords;
}

__device__ __forceinline__ void peer_put(unsigned long long* word, unsigned half, unsigned tag) {
    const unsigned long long v = (static_cast<unsigned long long>(tag) << 32) | half;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(word), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long peer_get(const unsigned long long* word) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(word) : "memory");
    return v;
}

// A value as its 32-bit halves (one for a float) and back.
__device__ __forceinline__ void peer_halves(double x, unsigned* h) {
    const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(x));
    h[0] = static_cast<unsigned>(b);
    h[1] = static_cast<unsigned>(b >> 32);
}
__device__ __forceinline__ void peer_halves(float x, unsigned* h) { h[0] = __float_as_uint(x); }
__device__ __forceinline__ void peer_join(const unsigned* h, double& x) {
    x = __longlong_as_double(static_cast<long long>((static_cast<unsigned long long>(h[1]) << 32) | h[0]));
}
__device__ __forceinline__ void peer_join(const unsigned* h, float& x) { x = __uint_as_float(h[0]); }

// One block per column: this rank's pairwise levels over its leaves (in place,
// as tree_kernel), the root published to every rank, then the ranks' roots
// folded in rank order -- the levels tree_kernel runs over world * leaves
// leaves once each rank's own leaves are joined.
template <class T, int OP>
__global__ void __launch_bounds__(1024) peer_finish_kernel(T* leaf_hi, T* leaf_comp, long long leaves, PeerAreas peers,
                                                          int rank, int world, unsigned long long seq,
                                                          unsigned long long limit_ns, T* out) {
    constexpr int H = sizeof(T) / 4;           // halves a value
    const int col = blockIdx.x;
    T* h = leaf_hi + col * leaves;
    T* c = leaf_comp + col * leaves;
    for (long long st = 1; st < leaves; st <<= 1) {
        for (long long idx = static_cast<long long>(threadIdx.x) * 2 * st; idx < leaves;
             idx += static_cast<long long>(blockDim.x) * 2 * st) {
            if (idx + st < leaves) {
                T a = h[idx], ac = c[idx];
                hk::ss::tree_join<OP>(a, ac, h[idx + st], c[idx + st]);
                h[idx] = a;
                c[idx] = ac;
            }
        }
        __syncthreads();
    }
    const int parity = static_cast<int>(seq & 1ull);
    const unsigned tag = static_cast<unsigned>(seq);
    unsigned char* const mine = peers.area[rank];
    __shared__ int missing;
    __shared__ T roots[kPeerRanks], comps[kPeerRanks];
    if (threadIdx.x == 0) missing = 0;
    __syncthreads();
    const int j = static_cast<int>(threadIdx.x);
    if (j < world) {
        // publish this rank's root into rank j's area: every half with the tag
        unsigned mh[2] = {0u, 0u}, mc[2] = {0u, 0u};
        peer_halves(h[0], mh);
        peer_halves(c[0], mc);
        unsigned long long* w = peer_words(peers.area[j], parity, rank, col);
        for (int k = 0; k < H; ++k) {
            peer_put(w + k, mh[k], tag);
            peer_put(w + 2 + k, mc[k], tag);
        }
        // rank j's root of this round from this rank's area
        const unsigned long long* r = peer_words(mine, parity, j, col);
        unsigned rh[2] = {0u, 0u}, rc[2] = {0u, 0u};
        bool up = false;
        unsigned long long t0 = 0;
        for (bool first = true;; first = false) {
            up = true;
            for (int k = 0; k < H; ++k) {
                const unsigned long long a = peer_get(r + k), b = peer_get(r + 2 + k);
                up = up && static_cast<unsigned>(a >> 32) == tag && static_cast<unsigned>(b >> 32) == tag;
                rh[k] = static_cast<unsigned>(a);
                rc[k] = static_cast<unsigned>(b);
            }
            if (up) break;
            if (first) t0 = peer_now();
            else if (peer_now() - t0 > limit_ns) break;
        }
        if (up) {
            peer_join(rh, roots[j]);
            peer_join(rc, comps[j]);
        } else {
            atomicAdd(&missing, 1);
            atomicOr(reinterpret_cast<unsigned*>(mine), HKB_PEER_TIMEOUT);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && missing == 0) {
        T v[kPeerRanks], vc[kPeerRanks];
        for (int r = 0; r < world; ++r) {
            v[r] = roots[r];
            vc[r] = comps[r];
        }
        for (int st = 1; st < world; st <<= 1)
            for (int idx = 0; idx + st < world; idx += 2 * st) hk::ss::tree_join<OP>(v[idx], vc[idx], v[idx + st], vc[idx + st]);
        out[col] = (OP == hk::ss::kSum) ? (hk::ss::finite(v[0]) ? v[0] + vc[0] : v[0]) : v[0];
    }
}

}  // namespace

struct hkb_peer {
    int device = 0, rank = 0, world = 1, dtype = HKB_F64, ncols = 1;
    unsigned char* mine = nullptr;
    PeerAreas areas{};
    bool opened[kPeerRanks] = {};
};

extern "C" {

int hkb_peer_create(int device, int rank, int world, int dtype, int ncols, hkb_peer** out, void* handle_out) {
    if (out == nullptr || handle_out == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_peer_create: null output");
    *out = nullptr;
    if (world < 1 || world > kPeerRanks || rank < 0 || rank >= world)
        return fail(HKB_ERR_RANGE, "rank %d of world %d: the peer finish takes 1..%d ranks", rank, world, kPeerRanks);
    if (dtype != HKB_F64 && dtype != HKB_F32) return fail(HKB_ERR_ARGUMENT, "unknown dtype %d", dtype);
    if (ncols < 1 || ncols > kMaxCols) return fail(HKB_ERR_RANGE, "ncols %d is outside 1..%d", ncols, kMaxCols);
    DeviceScope scope(device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    hkb_peer* p = new (std::nothrow) hkb_peer();
    if (p == nullptr) return fail(HKB_ERR_ARGUMENT, "out of host memory");
    p->device = device;
    p->rank = rank;
    p->world = world;
    p->dtype = dtype;
    p->ncols = ncols;
    cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&p->mine), kPeerAreaBytes);
    if (err == cudaSuccess) err = cudaMemset(p->mine, 0, kPeerAreaBytes);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    cudaIpcMemHandle_t handle;
    if (err == cudaSuccess) err = cudaIpcGetMemHandle(&handle, p->mine);
    if (err != cudaSuccess) {
        if (p->mine != nullptr) cudaFree(p->mine);
        delete p;
        return cuda_fail(err, "making the exchange area");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == HKB_PEER_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &handle, sizeof handle);
    p->areas.area[rank] = p->mine;
    *out = p;
    return HKB_OK;
}

int hkb_peer_connect(hkb_peer* peer, const void* handles) {
    if (peer == nullptr || handles == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_peer_connect: null argument");
    DeviceScope scope(peer->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    for (int r = 0; r < peer->world; ++r) {
        if (r == peer->rank || peer->opened[r]) continue;
        cudaIpcMemHandle_t handle;
        std::memcpy(&handle, static_cast<const char*>(handles) + static_cast<size_t>(r) * HKB_PEER_HANDLE_BYTES,
                    sizeof handle);
        void* ptr = nullptr;
        const cudaError_t err = cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) return fail(HKB_ERR_CUDA, "opening rank %d's exchange area: %s (%s)", r,
                                            cudaGetErrorString(err), cudaGetErrorName(err));
        peer->areas.area[r] = static_cast<unsigned char*>(ptr);
        peer->opened[r] = true;
    }
    return HKB_OK;
}

int hkb_peer_finish(hkb_peer* peer, int op, void* leaf_hi, void* leaf_comp, int64_t leaves, void* out,
                    uint64_t seq, uint64_t timeout_ns, void* stream) {
    if (peer == nullptr || leaf_hi == nullptr || leaf_comp == nullptr || out == nullptr)
        return fail(HKB_ERR_ARGUMENT, "hkb_peer_finish: null argument");
    int status = check_cells(op, peer->dtype, peer->ncols);
    if (status != HKB_OK) return status;
    if (leaves < 1) return fail(HKB_ERR_RANGE, "a tree needs at least one leaf");
    if ((seq & 0xffffffffull) == 0)
        return fail(HKB_ERR_ARGUMENT, "hkb_peer_finish: round %llu has a zero tag (rounds are numbered from 1 and "
                    "skip multiples of 2^32)", (unsigned long long)seq);
    for (int r = 0; r < peer->world; ++r)
        if (peer->areas.area[r] == nullptr)
            return fail(HKB_ERR_ARGUMENT, "rank %d's exchange area is not connected (hkb_peer_connect)", r);
    DeviceScope scope(peer->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    const unsigned long long limit = timeout_ns ? timeout_ns : kPeerWaitNs;
    auto s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(peer->ncols));
    const long long n = leaves;
    const int rk = peer->rank, w = peer->world;
    if (peer->dtype == HKB_F64) {
        double* h = static_cast<double*>(leaf_hi);
        double* c = static_cast<double*>(leaf_comp);
        double* o = static_cast<double*>(out);
        switch (op) {
            case HKB_OP_SUM: peer_finish_kernel<double, hk::ss::kSum><<<grid, 1024, 0, s>>>(h, c, n, peer->areas, rk, w, seq, limit, o); break;
            case HKB_OP_MAX: peer_finish_kernel<double, hk::ss::kMax><<<grid, 1024, 0, s>>>(h, c, n, peer->areas, rk, w, seq, limit, o); break;
            default: peer_finish_kernel<double, hk::ss::kMin><<<grid, 1024, 0, s>>>(h, c, n, peer->areas, rk, w, seq, limit, o); break;
        }
    } else {
        float* h = static_cast<float*>(leaf_hi);
        float* c = static_cast<float*>(leaf_comp);
        float* o = static_cast<float*>(out);
        switch (op) {
            case HKB_OP_SUM: peer_finish_kernel<float, hk::ss::kSum><<<grid, 1024, 0, s>>>(h, c, n, peer->areas, rk, w, seq, limit, o); break;
            case HKB_OP_MAX: peer_finish_kernel<float, hk::ss::kMax><<<grid, 1024, 0, s>>>(h, c, n, peer->areas, rk, w, seq, limit, o); break;
            default: peer_finish_kernel<float, hk::ss::kMin><<<grid, 1024, 0, s>>>(h, c, n, peer->areas, rk, w, seq, limit, o); break;
        }
    }
    HKB_CUDA(cudaGetLastError(), "launching the peer finish");
    return HKB_OK;
}

int hkb_peer_status(hkb_peer* peer, unsigned* flags) {
    if (peer == nullptr || flags == nullptr) return fail(HKB_ERR_ARGUMENT, "hkb_peer_status: null argument");
    *flags = 0;
    DeviceScope scope(peer->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "selecting the device");
    HKB_CUDA(cudaMemcpy(flags, peer->mine, sizeof(unsigned), cudaMemcpyDeviceToHost), "reading the exchange status");
    HKB_CUDA(cudaMemset(peer->mine, 0, sizeof(unsigned)), "clearing the exchange status");
    return HKB_OK;
}

void hkb_peer_free(hkb_peer* peer) {
    if (peer == nullptr) return;
    DeviceScope scope(peer->device);
    for (int r = 0; r < kPeerRanks; ++r)
        if (peer->opened[r]) cudaIpcCloseMemHandle(peer->areas.area[r]);
    if (peer->mine != nullptr) cudaFree(peer->mine);
    delete peer;
}

}  // extern "C"
