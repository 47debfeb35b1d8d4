// Run-time compilation of model-specialized rollout kernels.
//
// pz_spec.h writes, for one packed model, a translation unit whose body
// tables are literal; this file compiles it with NVRTC for the device in use,
// loads the cubin as a module, sizes its launch like the generic variants'
// (pick_launch) and launches it with the generic kernel's argument block.
// The kernel source itself (stepper_kernels.cuh and its headers) is carried
// inside the library as text (pz_spec_headers.inc, written by the build), so
// the library needs no source tree at run time, only libnvrtc.
//
// NVRTC is loaded on first use (libnvrtc.so.12, or the file PHYZB_NVRTC
// names); the driver calls come through the runtime's entry-point query, so
// the library links neither. Compiled cubins are kept per process and, unless
// PHYZB_KERNEL_CACHE is "0", in a cache directory keyed by a hash of the
// compiler version, the options, the generated source and the headers.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "pz_launch.h"
#include "pz_spec.h"
#include "pz_variants.h"
#include "pz_spec_headers.inc"

namespace pz {

struct SpecKernel {
    CUmodule mod = nullptr;
    CUfunction fn = nullptr;
    int static_smem = 0;
    int users = 0;                 // simulators running it
    unsigned long long stamp = 0;  // last lookup (least recently used goes first)
};

namespace {

constexpr int kSpecHeaderCount = (int)(sizeof(kSpecHeaderNames) / sizeof(kSpecHeaderNames[0]));

struct Nvrtc {
    decltype(&::nvrtcVersion) version = nullptr;
    decltype(&::nvrtcCreateProgram) create = nullptr;
    decltype(&::nvrtcDestroyProgram) destroy = nullptr;
    decltype(&::nvrtcAddNameExpression) add_name = nullptr;
    decltype(&::nvrtcCompileProgram) compile = nullptr;
    decltype(&::nvrtcGetProgramLogSize) log_size = nullptr;
    decltype(&::nvrtcGetProgramLog) log = nullptr;
    decltype(&::nvrtcGetCUBINSize) cubin_size = nullptr;
    decltype(&::nvrtcGetCUBIN) cubin = nullptr;
    decltype(&::nvrtcGetLoweredName) lowered = nullptr;
    decltype(&::nvrtcGetErrorString) error_string = nullptr;
    std::string error;  // empty: loaded
    std::string tag;    // "nvrtc <major>.<minor>"
};

template <class F>
bool sym(void* h, const char* name, F* f, std::string* err) {
    *f = reinterpret_cast<F>(dlsym(h, name));
    if (!*f) *err = std::string("libnvrtc has no ") + name;
    return *f != nullptr;
}

Nvrtc load_nvrtc() {
    Nvrtc n;
    void* h = nullptr;
    std::string tried;
    const char* env = getenv("PHYZB_NVRTC");
    const char* names[] = {env, "libnvrtc.so.12", "libnvrtc.so"};
    for (const char* name : names) {
        if (!name || !*name) continue;
        h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
        if (h) break;
        const char* e = dlerror();
        tried += std::string(tried.empty() ? "" : "; ") + (e ? e : name);
    }
    if (!h) {
        n.error = "model-specialized kernels need the CUDA runtime compiler (libnvrtc.so.12): " + tried;
        return n;
    }
    if (!sym(h, "nvrtcVersion", &n.version, &n.error) || !sym(h, "nvrtcCreateProgram", &n.create, &n.error) ||
        !sym(h, "nvrtcDestroyProgram", &n.destroy, &n.error) ||
        !sym(h, "nvrtcAddNameExpression", &n.add_name, &n.error) ||
        !sym(h, "nvrtcCompileProgram", &n.compile, &n.error) ||
        !sym(h, "nvrtcGetProgramLogSize", &n.log_size, &n.error) ||
        !sym(h, "nvrtcGetProgramLog", &n.log, &n.error) || !sym(h, "nvrtcGetCUBINSize", &n.cubin_size, &n.error) ||
        !sym(h, "nvrtcGetCUBIN", &n.cubin, &n.error) || !sym(h, "nvrtcGetLoweredName", &n.lowered, &n.error) ||
        !sym(h, "nvrtcGetErrorString", &n.error_string, &n.error))
        return n;
    int major = 0, minor = 0;
    n.version(&major, &minor);
    n.tag = "nvrtc " + std::to_string(major) + "." + std::to_string(minor);
    return n;
}

const Nvrtc& nvrtc() {
    static const Nvrtc n = load_nvrtc();
    return n;
}

struct Driver {
    decltype(&::cuModuleLoadData) load = nullptr;
    decltype(&::cuModuleGetFunction) get = nullptr;
    decltype(&::cuFuncGetAttribute) attr = nullptr;
    decltype(&::cuFuncSetAttribute) set_attr = nullptr;
    decltype(&::cuOccupancyMaxActiveBlocksPerMultiprocessor) occupancy = nullptr;
    decltype(&::cuLaunchKernel) launch = nullptr;
    decltype(&::cuModuleUnload) unload = nullptr;
    std::string error;
};

template <class F>
bool entry(const char* name, F* f, std::string* err) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || !p) {
        *err = std::string("driver entry point ") + name + " unavailable (" + cudaGetErrorString(e) + ")";
        return false;
    }
    *f = reinterpret_cast<F>(p);
    return true;
}

Driver load_driver() {
    Driver d;
    if (!entry("cuModuleLoadData", &d.load, &d.error) || !entry("cuModuleGetFunction", &d.get, &d.error) ||
        !entry("cuFuncGetAttribute", &d.attr, &d.error) || !entry("cuFuncSetAttribute", &d.set_attr, &d.error) ||
        !entry("cuOccupancyMaxActiveBlocksPerMultiprocessor", &d.occupancy, &d.error) ||
        !entry("cuLaunchKernel", &d.launch, &d.error) || !entry("cuModuleUnload", &d.unload, &d.error))
        return d;
    return d;
}

const Driver& driver() {
    static const Driver d = load_driver();
    return d;
}

std::string cu_error(const char* what, CUresult r) {
    return std::string(what) + " failed (CUresult " + std::to_string((int)r) + ")";
}

// FNV-1a, 64 bit, over a sequence of strings (each followed by a 0 byte)
struct Hash {
    uint64_t h;
    explicit Hash(uint64_t seed) : h(seed) {}
    void add(const std::string& s) {
        for (unsigned char c : s) h = (h ^ c) * 0x100000001b3ull;
        h = (h ^ 0u) * 0x100000001b3ull;
    }
};

std::string cache_dir() {
    const char* env = getenv("PHYZB_KERNEL_CACHE");
    if (env && std::strcmp(env, "0") == 0) return "";
    if (env && *env) return env;
    const char* home = getenv("HOME");
    if (!home || !*home) return "";
    return std::string(home) + "/.cache/phyzb";
}

void make_dirs(const std::string& dir) {
    for (size_t i = 1; i <= dir.size(); i++)
        if (i == dir.size() || dir[i] == '/') mkdir(dir.substr(0, i).c_str(), 0755);
}

// cache file: "PZSPEC1\n<lowered name>\n" then the cubin
bool read_cached(const std::string& path, std::string* lowered, std::vector<char>* cubin) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    std::vector<char> all;
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) all.insert(all.end(), buf, buf + n);
    std::fclose(f);
    const std::string magic = "PZSPEC1\n";
    if (all.size() < magic.size() || std::memcmp(all.data(), magic.data(), magic.size()) != 0) return false;
    size_t i = magic.size();
    while (i < all.size() && all[i] != '\n') i++;
    if (i >= all.size()) return false;
    lowered->assign(all.data() + magic.size(), all.data() + i);
    cubin->assign(all.begin() + (long)i + 1, all.end());
    return !cubin->empty();
}

void write_cached(const std::string& dir, const std::string& path, const std::string& lowered,
                  const std::vector<char>& cubin) {
    make_dirs(dir);
    const std::string tmp = path + ".tmp" + std::to_string((long long)getpid());
    FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) return;
    const std::string head = "PZSPEC1\n" + lowered + "\n";
    const bool ok = std::fwrite(head.data(), 1, head.size(), f) == head.size() &&
                    std::fwrite(cubin.data(), 1, cubin.size(), f) == cubin.size();
    std::fclose(f);
    if (ok)
        std::rename(tmp.c_str(), path.c_str());
    else
        std::remove(tmp.c_str());
}

cudaError_t compile(const std::string& src, const std::string& name, const std::vector<std::string>& opts,
                    std::string* lowered, std::vector<char>* cubin, std::string* err) {
    const Nvrtc& n = nvrtc();
    if (!n.error.empty()) {
        *err = n.error;
        return cudaErrorNotSupported;
    }
    nvrtcProgram prog = nullptr;
    nvrtcResult r = n.create(&prog, src.c_str(), "pz_spec_rollout.cu", kSpecHeaderCount, kSpecHeaderTexts,
                             kSpecHeaderNames);
    if (r != NVRTC_SUCCESS) {
        *err = std::string("nvrtcCreateProgram: ") + n.error_string(r);
        return cudaErrorUnknown;
    }
    std::vector<const char*> o;
    for (const std::string& s : opts) o.push_back(s.c_str());
    r = n.add_name(prog, name.c_str());
    if (r == NVRTC_SUCCESS) r = n.compile(prog, (int)o.size(), o.data());
    if (r != NVRTC_SUCCESS) {
        size_t ls = 0;
        n.log_size(prog, &ls);
        std::string log(ls, '\0');
        if (ls) n.log(prog, &log[0]);
        *err = std::string("runtime compile of the specialized rollout kernel failed: ") + n.error_string(r) +
               "\n" + log;
        n.destroy(&prog);
        return cudaErrorUnknown;
    }
    const char* low = nullptr;
    size_t cs = 0;
    r = n.lowered(prog, name.c_str(), &low);
    if (r == NVRTC_SUCCESS) *lowered = low;
    if (r == NVRTC_SUCCESS) r = n.cubin_size(prog, &cs);
    if (r == NVRTC_SUCCESS) {
        cubin->resize(cs);
        r = n.cubin(prog, cubin->data());
    }
    n.destroy(&prog);
    if (r != NVRTC_SUCCESS || cubin->empty()) {
        *err = std::string("runtime compile produced no cubin: ") + n.error_string(r);
        return cudaErrorUnknown;
    }
    return cudaSuccess;
}

std::mutex g_mu;
std::map<std::string, std::unique_ptr<SpecKernel>> g_kernels;  // key: device + source hash
unsigned long long g_clock = 0;

// Unload modules no simulator holds, oldest lookup first, until at most
// kSpecModuleCap stay loaded (caller holds g_mu). A module's device is the
// one current at its load; the key's prefix names it.
int module_cap() {
    static const int cap = [] {
        const char* e = getenv("PHYZB_SPEC_MODULE_CAP");  // tests shrink it
        const int v = e ? atoi(e) : 0;
        return v > 0 ? v : kSpecModuleCap;
    }();
    return cap;
}

void trim_locked() {
    const Driver& drv = driver();
    while ((int)g_kernels.size() > module_cap()) {
        auto victim = g_kernels.end();
        for (auto it = g_kernels.begin(); it != g_kernels.end(); ++it)
            if (it->second->users == 0 && (victim == g_kernels.end() || it->second->stamp < victim->second->stamp))
                victim = it;
        if (victim == g_kernels.end()) return;  // every loaded module is in use
        int dev = 0, cur = 0;
        dev = std::atoi(victim->first.c_str());
        cudaGetDevice(&cur);
        if (dev != cur) cudaSetDevice(dev);
        if (drv.unload) drv.unload(victim->second->mod);
        if (dev != cur) cudaSetDevice(cur);
        g_kernels.erase(victim);
    }
}

// The module of `src` on the current device: from this process's table,
// else the disk cache, else a fresh compile.
cudaError_t get_kernel(const std::string& src, const std::string& name, SpecKernel** out, std::string* err) {
    const Driver& drv = driver();
    if (!drv.error.empty()) {
        *err = drv.error;
        return cudaErrorNotSupported;
    }
    int dev = 0, major = 0, minor = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return e;
    }
    // the kernel's Tensor Memory and bulk-copy instructions are sm_100a's;
    // PHYZB_SPEC_NVRTC_OPTS appends options (space-separated) for tuning
    std::vector<std::string> opts = {"-arch=sm_" + std::to_string(major * 10 + minor) + "a", "-std=c++17",
                                     "-lineinfo"};
    if (const char* extra = getenv("PHYZB_SPEC_NVRTC_OPTS")) {
        std::string tok;
        for (const char* c = extra;; c++) {
            if (*c == ' ' || *c == '\0') {
                if (!tok.empty()) opts.push_back(tok);
                tok.clear();
                if (*c == '\0') break;
            } else {
                tok += *c;
            }
        }
    }
    Hash h1(0xcbf29ce484222325ull), h2(0x84222325cbf29ce4ull);
    for (Hash* h : {&h1, &h2}) {
        h->add(nvrtc().tag);
        for (const std::string& s : opts) h->add(s);
        h->add(name);
        h->add(src);
        for (int k = 0; k < kSpecHeaderCount; k++) h->add(kSpecHeaderTexts[k]);
    }
    char hex[40];
    std::snprintf(hex, sizeof hex, "%016llx%016llx", (unsigned long long)h1.h, (unsigned long long)h2.h);
    const std::string key = std::to_string(dev) + ":" + hex;
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_kernels.find(key);
    if (it != g_kernels.end()) {
        it->second->stamp = ++g_clock;
        *out = it->second.get();
        return cudaSuccess;
    }
    const std::string dir = cache_dir();
    const std::string path = dir.empty() ? "" : dir + "/" + hex + ".cubin";
    std::string lowered;
    std::vector<char> cubin;
    bool cached = !path.empty() && read_cached(path, &lowered, &cubin);
    auto k = std::make_unique<SpecKernel>();
    for (int attempt = 0; attempt < 2; attempt++) {
        if (!cached) {
            if ((e = compile(src, name, opts, &lowered, &cubin, err)) != cudaSuccess) return e;
            if (!path.empty()) write_cached(dir, path, lowered, cubin);
        }
        CUresult r = drv.load(&k->mod, cubin.data());
        if (r == CUDA_SUCCESS) r = drv.get(&k->fn, k->mod, lowered.c_str());
        if (r == CUDA_SUCCESS) break;
        if (!cached) {
            *err = cu_error("loading the specialized rollout kernel", r);
            return cudaErrorUnknown;
        }
        cached = false;  // a stale or damaged cache entry: compile afresh
    }
    CUresult r = drv.attr(&k->static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, k->fn);
    if (r != CUDA_SUCCESS) {
        *err = cu_error("cuFuncGetAttribute", r);
        return cudaErrorUnknown;
    }
    k->stamp = ++g_clock;
    *out = k.get();
    g_kernels.emplace(key, std::move(k));
    return cudaSuccess;
}

}  // namespace

void spec_retain(const SpecKernel* k) {
    if (!k) return;
    std::lock_guard<std::mutex> lock(g_mu);
    const_cast<SpecKernel*>(k)->users++;
    trim_locked();
}

void spec_release(const SpecKernel* k) {
    if (!k) return;
    std::lock_guard<std::mutex> lock(g_mu);
    SpecKernel* m = const_cast<SpecKernel*>(k);
    if (m->users > 0) m->users--;
    trim_locked();
}

namespace {

template <class T>
cudaError_t spec_compile(const SpecLayout& L, const RolloutArgs<T>& a, int W, SpecKernel** k, std::string* err,
                         bool sliced = false) {
    const std::string src = spec_source<T>(L.blob, L.off_bi, L.off_pd, L.off_pdmap, a.nb, a.nv, a.npd, W, sliced);
    return get_kernel(src, spec_kernel_name<T>(L.feat, L.tm), k, err);
}

cudaError_t fn_attr(const SpecKernel* k, CUfunction_attribute at, int* v, std::string* err) {
    const CUresult r = driver().attr(v, at, k->fn);
    if (r == CUDA_SUCCESS) return cudaSuccess;
    *err = cu_error("cuFuncGetAttribute", r);
    return cudaErrorUnknown;
}

// Launch shape of kernel k (compiled for W threads) on layout L, scored like
// the generic variants' (worlds resident per SM x fill of the last wave).
template <class T>
cudaError_t spec_config(const DeviceLimits& dl, const SpecKernel* k, const SpecLayout& L, const RolloutArgs<T>& a,
                        int W, LaunchCfg* cfg, std::string* err) {
    const int dyn_cap = dl.smem_optin - k->static_smem;
    const Driver& drv = driver();
    CUresult r = drv.set_attr(k->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, dyn_cap);
    if (r != CUDA_SUCCESS) {
        *err = cu_error("cuFuncSetAttribute", r);
        return cudaErrorUnknown;
    }
    CUfunction fn = k->fn;
    auto occupancy = [&drv, fn](int* blocks, int w, size_t smem) {
        return drv.occupancy(blocks, fn, w, smem) == CUDA_SUCCESS ? cudaSuccess : cudaErrorUnknown;
    };
    // the slice shape is that of the kernel's slice-mode twin (spec_sliced)
    const cudaError_t e = pick_launch(dl, dyn_cap, L.tm, (int)sizeof(T), L.scratch, L.bytes, a.nworld, L.tmem_cols,
                                      (int)TMEM_COLS, occupancy, cfg, W, W, true);
    if (e != cudaSuccess)
        *err = "the specialized rollout kernel does not launch with " + std::to_string(W) + " worlds per block";
    return e;
}

// The widest one-per-SM Tensor-Memory block that `regs` registers a thread,
// the layout's shared memory per world and its TMEM columns per world allow.
int tm_width_limit(const DeviceLimits& dl, int dyn_cap, int regs, int esz, const SpecLayout& L) {
    const int regs_warp = ((regs * 32 + 255) / 256) * 256;  // the register file's allocation unit
    int best = 0;
    for (int W = 32; W <= dl.max_threads; W += 32) {
        if ((W / 32) * regs_warp > dl.regs_per_sm) break;
        if ((long long)L.bytes + (long long)L.scratch * esz * W > dyn_cap) break;
        if (L.tmem_cols > tmem_cols_per_thread(W / 32, (int)TMEM_COLS)) break;
        best = W;
    }
    return best;
}

}  // namespace

template <class T>
cudaError_t spec_candidates(const SpecLayout* lays, int nlay, const RolloutArgs<T>& a,
                            std::vector<SpecChoice>* out, std::string* err) {
    int dev = 0;
    DeviceLimits dl{0, 0};
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&dl.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&dl.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&dl.regs_per_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&dl.max_threads, cudaDevAttrMaxThreadsPerBlock, dev)) != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return e;
    }
    out->clear();
    for (int li = 0; li < nlay; li++) {
        const SpecLayout& L = lays[li];
        SpecKernel* k = nullptr;
        if ((e = spec_compile<T>(L, a, L.w0, &k, err)) != cudaSuccess) return e;
        LaunchCfg c{};
        if ((e = spec_config<T>(dl, k, L, a, L.w0, &c, err)) != cudaSuccess) return e;
        out->push_back(SpecChoice{li, k, c});
        // a second width: Tensor-Memory tables as wide as the compiled
        // kernel's registers and the table's on-chip memory per world allow
        // (one block per SM); shared-memory tables at whole warps
        int w2 = 0;
        if (L.tm) {
            int regs = 0;
            if ((e = fn_attr(k, CU_FUNC_ATTRIBUTE_NUM_REGS, &regs, err)) != cudaSuccess) return e;
            const int wmax = tm_width_limit(dl, dl.smem_optin - k->static_smem, regs, (int)sizeof(T), L);
            LaunchCfg wide{};
            auto fits = [wmax](int* blocks, int w, size_t) {
                *blocks = w <= wmax ? 1 : 0;
                return cudaSuccess;
            };
            if (wmax > 0 && pick_launch(dl, dl.smem_optin - k->static_smem, true, (int)sizeof(T), L.scratch, L.bytes,
                                        a.nworld, L.tmem_cols, (int)TMEM_COLS, fits, &wide, 0, wmax) == cudaSuccess)
                w2 = wide.W;
        } else {
            w2 = (L.w0 / 32) * 32;
        }
        if (w2 > 0 && w2 != L.w0) {
            SpecKernel* k2 = nullptr;
            std::string e2;
            LaunchCfg c2{};
            if (spec_compile<T>(L, a, w2, &k2, &e2) == cudaSuccess &&
                spec_config<T>(dl, k2, L, a, w2, &c2, &e2) == cudaSuccess)
                out->push_back(SpecChoice{li, k2, c2});
            cudaGetLastError();  // a width that does not launch is simply not a candidate
        }
    }
    if (out->empty()) {
        *err = "no table layout to specialize";
        return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

template <class T>
cudaError_t spec_sliced(const SpecLayout& L, const RolloutArgs<T>& a, int W, const SpecKernel** out,
                        std::string* err) {
    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) {
        *err = cudaGetErrorString(e);
        return e;
    }
    SpecKernel* k = nullptr;
    if ((e = spec_compile<T>(L, a, W, &k, err, true)) != cudaSuccess) return e;
    const CUresult r = driver().set_attr(k->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, optin - k->static_smem);
    if (r != CUDA_SUCCESS) {
        *err = cu_error("cuFuncSetAttribute", r);
        return cudaErrorUnknown;
    }
    *out = k;
    return cudaSuccess;
}

template <class T>
cudaError_t spec_launch(const SpecKernel* k, const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s) {
    if (a.nsteps <= 0 || a.nworld <= 0) return cudaSuccess;
    RolloutArgs<T> args = a;
    void* params[] = {&args};
    const CUresult r = driver().launch(k->fn, (unsigned)cfg.grid, 1, 1, (unsigned)cfg.W, 1, 1, (unsigned)cfg.smem,
                                       (CUstream)s, params, nullptr);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorLaunchFailure;
}

template cudaError_t spec_candidates<float>(const SpecLayout*, int, const RolloutArgs<float>&,
                                            std::vector<SpecChoice>*, std::string*);
template cudaError_t spec_candidates<double>(const SpecLayout*, int, const RolloutArgs<double>&,
                                             std::vector<SpecChoice>*, std::string*);
template cudaError_t spec_sliced<float>(const SpecLayout&, const RolloutArgs<float>&, int, const SpecKernel**,
                                        std::string*);
template cudaError_t spec_sliced<double>(const SpecLayout&, const RolloutArgs<double>&, int, const SpecKernel**,
                                         std::string*);
template cudaError_t spec_launch<float>(const SpecKernel*, const RolloutArgs<float>&, const LaunchCfg&, cudaStream_t);
template cudaError_t spec_launch<double>(const SpecKernel*, const RolloutArgs<double>&, const LaunchCfg&,
                                         cudaStream_t);

}  // namespace pz
