// tile_jit.cu -- a tile graph's specialised kernel: the lowered program
// (tile.cu) written out as compile-time constants, compiled for sm_100a at
// run time by NVRTC and cached per device and program.
//
// The reference compiles every distinct graph with NVRTC (tile/run.go:40,
// kernels cached by source). Here the compiled code is not a new rendering
// of the graph: it is tile_kernel.cuh's own kernel body, tile_body<BULK, G,
// S>, instantiated with a struct S that holds the program's instructions and
// window descriptors as constants (interpret_s), so every instruction's
// decode, dispatch and operand addressing folds away and the windows' taps
// are parameter-bank operands, while each value is computed by the same
// device functions in the same order as the interpreter: the two produce
// the same bits. The device headers travel inside the library (rtc_headers.inc,
// written by build.py); NVRTC is opened with dlopen on first use and the
// module loaded through the runtime's driver entry points, so the library
// links against neither.
//
// A streaming reduction (k_red_direct) is specialised the same way: its
// chain of steps compiled in as constants (get_chain), the kernel named by
// its template instance (an NVRTC name expression).
//
// Modes (simtgo_tile_set_jit, or SIMTGO_TILE_JIT in the environment at the
// first tile launch): 0 = the interpreter only; 1 (default) = specialise
// every program tile.cu routes here (up to 32 instructions), falling back to
// the interpreter when NVRTC cannot be opened (libnvrtc.so.12, or the
// library SIMTGO_NVRTC_LIB names); 2 = specialise or fail. A program whose
// compilation fails is an error in modes 1 and 2 (it is a bug, not a
// missing dependency).
//
// Compiled cubins are also kept on disk (internal/jit/diskcache.go keeps the
// reference's PTX the same way), so a new process does not compile again:
// in $SIMTGO_B200_CACHE, else $XDG_CACHE_HOME/simtgo_b200, else
// ~/.cache/simtgo_b200 ("off" disables it). An entry is named by a hash of
// everything that can change its bytes -- the source with the embedded
// headers, the compile options and NVRTC's version -- and holds that whole
// identity before the cubin, so a read serves the cubin only when the
// identity matches byte for byte: a hash collision is a miss, never a wrong
// kernel. Every failure to read or write is a miss.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "tile_kernel.cuh"
#include "tile_jit.h"

namespace {

#include "rtc_headers.inc"  // kRtcHeaderNames[], kRtcHeaderSources[], kRtcHeaderCount

// ---- NVRTC, opened on first use ----------------------------------------------
typedef int nvrtcResult_t;
typedef struct _nvrtcProgram* nvrtcProgram_t;
struct Nvrtc {
    nvrtcResult_t (*create)(nvrtcProgram_t*, const char*, const char*, int, const char* const*,
                            const char* const*);
    nvrtcResult_t (*compile)(nvrtcProgram_t, int, const char* const*);
    nvrtcResult_t (*log_size)(nvrtcProgram_t, size_t*);
    nvrtcResult_t (*log)(nvrtcProgram_t, char*);
    nvrtcResult_t (*cubin_size)(nvrtcProgram_t, size_t*);
    nvrtcResult_t (*cubin)(nvrtcProgram_t, char*);
    nvrtcResult_t (*destroy)(nvrtcProgram_t*);
    const char* (*err)(nvrtcResult_t);
    nvrtcResult_t (*version)(int*, int*);
    nvrtcResult_t (*add_name)(nvrtcProgram_t, const char*);
    nvrtcResult_t (*lowered)(nvrtcProgram_t, const char*, const char**);
    bool ok = false;
    std::string why;
};

Nvrtc g_rtc;
std::once_flag g_rtc_once;

// SIMTGO_NVRTC_LIB names the library to open instead of libnvrtc.so.12
// (a path, or a name the loader searches for).
void open_nvrtc() {
    const char* want = getenv("SIMTGO_NVRTC_LIB");
    void* h = nullptr;
    if (want && *want) {
        h = dlopen(want, RTLD_NOW | RTLD_LOCAL);
    } else {
        h = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnvrtc.so", RTLD_NOW | RTLD_LOCAL);
    }
    if (!h) {
        const char* e = dlerror();
        g_rtc.why = std::string(want && *want ? want : "libnvrtc.so.12") +
                    " could not be opened: " + (e ? e : "?");
        return;
    }
    bool all = true;
    auto sym = [&](const char* name) {
        void* p = dlsym(h, name);
        all = all && p;
        return p;
    };
    g_rtc.create = (decltype(g_rtc.create))sym("nvrtcCreateProgram");
    g_rtc.compile = (decltype(g_rtc.compile))sym("nvrtcCompileProgram");
    g_rtc.log_size = (decltype(g_rtc.log_size))sym("nvrtcGetProgramLogSize");
    g_rtc.log = (decltype(g_rtc.log))sym("nvrtcGetProgramLog");
    g_rtc.cubin_size = (decltype(g_rtc.cubin_size))sym("nvrtcGetCUBINSize");
    g_rtc.cubin = (decltype(g_rtc.cubin))sym("nvrtcGetCUBIN");
    g_rtc.destroy = (decltype(g_rtc.destroy))sym("nvrtcDestroyProgram");
    g_rtc.err = (decltype(g_rtc.err))sym("nvrtcGetErrorString");
    g_rtc.version = (decltype(g_rtc.version))sym("nvrtcVersion");
    g_rtc.add_name = (decltype(g_rtc.add_name))sym("nvrtcAddNameExpression");
    g_rtc.lowered = (decltype(g_rtc.lowered))sym("nvrtcGetLoweredName");
    if (!all) {
        g_rtc.why = "libnvrtc.so.12 lacks an entry point this library needs";
        return;
    }
    g_rtc.ok = true;
}

// ---- driver entry points ------------------------------------------------------
struct Drv {
    CUresult (*load)(CUmodule*, const void*);
    CUresult (*get_fn)(CUfunction*, CUmodule, const char*);
    CUresult (*set_attr)(CUfunction, CUfunction_attribute, int);
    CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                       unsigned, CUstream, void**, void**);
    CUresult (*occupancy)(int*, CUfunction, int, size_t);
    CUresult (*err)(CUresult, const char**);
    CUresult (*unload)(CUmodule);
    bool ok = false;
};
Drv g_drv;
std::once_flag g_drv_once;

void open_driver() {
    bool all = true;
    auto ep = [&](const char* name) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        all = all && fn;
        return fn;
    };
    g_drv.load = (decltype(g_drv.load))ep("cuModuleLoadData");
    g_drv.get_fn = (decltype(g_drv.get_fn))ep("cuModuleGetFunction");
    g_drv.set_attr = (decltype(g_drv.set_attr))ep("cuFuncSetAttribute");
    g_drv.launch = (decltype(g_drv.launch))ep("cuLaunchKernel");
    g_drv.occupancy = (decltype(g_drv.occupancy))ep("cuOccupancyMaxActiveBlocksPerMultiprocessor");
    g_drv.err = (decltype(g_drv.err))ep("cuGetErrorString");
    g_drv.unload = (decltype(g_drv.unload))ep("cuModuleUnload");
    g_drv.ok = all;
}

int drv_status(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return 0;
    const char* s = nullptr;
    if (g_drv.err) g_drv.err(r, &s);
    return sg::fail(SIMTGO_EDEVICE, "tile: %s failed: %s (CUresult %d)", what, s ? s : "?",
                    (int)r);
}

// ---- mode and counters --------------------------------------------------------
std::atomic<int> g_mode{-1};
std::atomic<int64_t> g_compiled{0}, g_launches{0}, g_disk_hits{0};

int mode() {
    int m = g_mode.load();
    if (m < 0) {
        const char* e = getenv("SIMTGO_TILE_JIT");
        int v = 1;
        if (e && (e[0] == '0' || e[0] == '1' || e[0] == '2') && e[1] == 0) v = e[0] - '0';
        int expect = -1;
        g_mode.compare_exchange_strong(expect, v);
        m = g_mode.load();
    }
    return m;
}

// The prelude every specialised source starts with: NVRTC has no C library
// headers, so the integer types and limits the device headers use come from
// here, and CUtensorMap (only named by tma.cuh's device helpers) is an
// opaque 128-byte type.
const char* kPrelude =
    "typedef signed char int8_t; typedef short int16_t; typedef int int32_t;\n"
    "typedef long long int64_t; typedef unsigned char uint8_t;\n"
    "typedef unsigned short uint16_t; typedef unsigned int uint32_t;\n"
    "typedef unsigned long long uint64_t; typedef unsigned long long uintptr_t;\n"
    "#define INT32_MAX 2147483647\n"
    "#define INT32_MIN (-2147483647 - 1)\n"
    "#define INT64_MAX 9223372036854775807LL\n"
    "struct alignas(64) CUtensorMap { unsigned long long opaque[16]; };\n";

struct Entry {
    CUmodule mod = nullptr;
    CUfunction fn = nullptr;
    int dev = -1;
};
std::mutex g_mu;
std::unordered_map<std::string, Entry> g_cache;  // key: device | source

const char* const kOptArch = "-arch=sm_100a";

// ---- the persistent cubin cache -------------------------------------------------
std::string cache_dir() {
    const char* e = getenv("SIMTGO_B200_CACHE");
    if (e && *e) return strcmp(e, "off") == 0 ? std::string() : std::string(e);
    if ((e = getenv("XDG_CACHE_HOME")) && *e) return std::string(e) + "/simtgo_b200";
    if ((e = getenv("HOME")) && *e) return std::string(e) + "/.cache/simtgo_b200";
    return std::string();
}

// What determines a cubin's bytes: options, NVRTC's version, the embedded
// headers and the source.
std::string identity(const std::string& src) {
    int major = 0, minor = 0;
    if (g_rtc.version) g_rtc.version(&major, &minor);
    std::string id = std::string("entry v2 ") + kOptArch + " -std=c++17 --fmad=false taps=" +
                     std::to_string(SIMTGO_TILE_MAX_TAPS) + " nvrtc " + std::to_string(major) +
                     "." + std::to_string(minor) + "\n";
    for (int i = 0; i < kRtcHeaderCount; i++) {
        id += kRtcHeaderNames[i];
        id += '\0';
        id += std::to_string(strlen(kRtcHeaderSources[i]));
        id += '\0';
        id += kRtcHeaderSources[i];
    }
    id += src;
    return id;
}

// 128 bits of FNV-1a (two 64-bit passes, different offset bases) as hex.
std::string name_of(const std::string& id) {
    uint64_t a = 0xcbf29ce484222325ull, b = 0x84222325cbf29ce4ull;
    for (unsigned char ch : id) {
        a = (a ^ ch) * 0x100000001b3ull;
        b = (b ^ ch) * 0x100000001b3ull;
    }
    char buf[40];
    snprintf(buf, sizeof buf, "%016llx%016llx", (unsigned long long)a, (unsigned long long)b);
    return buf;
}

bool read_all(const std::string& path, std::string* out) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    out->clear();
    char buf[1 << 16];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
    const bool ok = !ferror(f);
    fclose(f);
    return ok;
}

// A compiled entry: the cubin and its kernel's (lowered) name.
struct Compiled {
    std::string cubin, name;
};

// The cached entry of `id`, if one with exactly this identity exists. An
// entry is [u64 |id|][id][u64 |name|][name][cubin].
bool disk_read(const std::string& id, Compiled* c) {
    const std::string dir = cache_dir();
    if (dir.empty()) return false;
    std::string file;
    if (!read_all(dir + "/" + name_of(id) + ".cubin", &file)) return false;
    const uint64_t n = id.size();
    if (file.size() < 16 + n) return false;
    uint64_t stored = 0, nl = 0;
    memcpy(&stored, file.data(), 8);
    if (stored != n || file.compare(8, n, id) != 0) return false;
    memcpy(&nl, file.data() + 8 + n, 8);
    if (nl == 0 || file.size() <= 16 + n + nl) return false;
    c->name.assign(file, 16 + n, nl);
    c->cubin.assign(file, 16 + n + nl, std::string::npos);
    return true;
}

void disk_write(const std::string& id, const Compiled& c) {
    const std::string& cubin = c.cubin;
    std::string dir = cache_dir();
    if (dir.empty() || cubin.empty()) return;
    for (size_t i = 1; i <= dir.size(); i++)  // mkdir -p
        if (i == dir.size() || dir[i] == '/') mkdir(dir.substr(0, i).c_str(), 0755);
    const std::string path = dir + "/" + name_of(id) + ".cubin";
    // A temporary name of this writer's own (process and a per-process
    // count: threads of one process may write the same entry at once).
    static std::atomic<uint64_t> seq{0};
    const std::string tmp = path + ".tmp" + std::to_string((long)getpid()) + "." +
                            std::to_string(seq.fetch_add(1));
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f) return;
    const uint64_t n = id.size(), nl = c.name.size();
    bool ok = fwrite(&n, 8, 1, f) == 1 && fwrite(id.data(), 1, n, f) == n &&
              fwrite(&nl, 8, 1, f) == 1 && fwrite(c.name.data(), 1, nl, f) == nl &&
              fwrite(cubin.data(), 1, cubin.size(), f) == cubin.size();
    ok = fclose(f) == 0 && ok;
    if (!ok || rename(tmp.c_str(), path.c_str()) != 0) unlink(tmp.c_str());
}

// Compiles src; its kernel is the extern "C" function `name`, or, with
// expr, the template instance the name expression expr denotes.
int compile_source(const std::string& src, const char* name, const char* expr, Compiled* out) {
    std::string* cubin = &out->cubin;
    nvrtcProgram_t prog = nullptr;
    nvrtcResult_t r = g_rtc.create(&prog, src.c_str(), "tile_spec.cu", kRtcHeaderCount,
                                   kRtcHeaderSources, kRtcHeaderNames);
    if (r) return sg::fail(SIMTGO_EDEVICE, "tile: nvrtcCreateProgram: %s", g_rtc.err(r));
    if (expr && (r = g_rtc.add_name(prog, expr))) {
        g_rtc.destroy(&prog);
        return sg::fail(SIMTGO_EDEVICE, "tile: nvrtcAddNameExpression: %s", g_rtc.err(r));
    }
    const std::string taps = "-DSIMTGO_TILE_MAX_TAPS=" + std::to_string(SIMTGO_TILE_MAX_TAPS);
    const char* opts[] = {kOptArch, "-std=c++17", "--fmad=false", taps.c_str()};
    r = g_rtc.compile(prog, 4, opts);
    if (r) {
        size_t n = 0;
        g_rtc.log_size(prog, &n);
        std::string log(n, '\0');
        if (n) g_rtc.log(prog, &log[0]);
        g_rtc.destroy(&prog);
        if (log.size() > 1500) log.resize(1500);
        return sg::fail(SIMTGO_EDEVICE, "tile: run-time compilation of the graph's kernel failed: "
                                        "%s\n%s",
                        g_rtc.err(r), log.c_str());
    }
    out->name = name ? name : "";
    if (expr) {
        const char* lowered = nullptr;
        if ((r = g_rtc.lowered(prog, expr, &lowered)) || !lowered) {
            g_rtc.destroy(&prog);
            return sg::fail(SIMTGO_EDEVICE, "tile: nvrtcGetLoweredName: %s", g_rtc.err(r));
        }
        out->name = lowered;
    }
    size_t n = 0;
    g_rtc.cubin_size(prog, &n);
    cubin->assign(n, '\0');
    if (n) g_rtc.cubin(prog, &(*cubin)[0]);
    g_rtc.destroy(&prog);
    return 0;
}

// The compiled entry for src (memory cache per device, then the disk cache,
// then NVRTC), loaded on the current device with its dynamic shared memory
// limit set to dyn_max. Returns nullptr with 0 when specialisation is off
// or (mode 1) NVRTC is unavailable.
int get_kernel(const std::string& src, const char* name, const char* expr, int dyn_max,
               CUfunction* out) {
    *out = nullptr;
    const int m = mode();
    if (m == 0) return 0;
    std::call_once(g_rtc_once, open_nvrtc);
    std::call_once(g_drv_once, open_driver);
    if (!g_rtc.ok || !g_drv.ok) {
        if (m == 1) return 0;
        return sg::fail(SIMTGO_EDEVICE, "tile: specialised kernels are required but %s",
                        !g_rtc.ok ? g_rtc.why.c_str()
                                  : "the driver's module entry points are not available");
    }
    int dev = -1;
    int rc = sg::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    const std::string key = std::to_string(dev) + "|" + src;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_cache.find(key);
        if (it != g_cache.end()) {
            *out = it->second.fn;
            return 0;
        }
    }
    // Not cached: read or compile, and load, without holding the lock, so
    // that launches of kernels already loaded do not wait for a compile. Two
    // threads that miss on the same program both build it; the first to
    // finish keeps its module and the other unloads its own.
    Compiled c;
    const std::string id = identity(src);
    if (disk_read(id, &c)) {
        g_disk_hits.fetch_add(1);
    } else {
        if ((rc = compile_source(src, name, expr, &c))) return rc;
        g_compiled.fetch_add(1);
        disk_write(id, c);
    }
    Entry e;
    e.dev = dev;
    if ((rc = drv_status(g_drv.load(&e.mod, c.cubin.data()), "cuModuleLoadData"))) return rc;
    if ((rc = drv_status(g_drv.get_fn(&e.fn, e.mod, c.name.c_str()), "cuModuleGetFunction")) ||
        (dyn_max > 0 &&
         (rc = drv_status(
              g_drv.set_attr(e.fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, dyn_max),
              "cuFuncSetAttribute")))) {
        if (g_drv.unload) g_drv.unload(e.mod);
        return rc;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto ins = g_cache.emplace(key, e);
    if (!ins.second && g_drv.unload) g_drv.unload(e.mod);  // another thread's came first
    *out = ins.first->second.fn;
    return 0;
}

}  // namespace

namespace tilejit {

std::string spec_source(const tilek::Program& P, const Form& f) {
    const bool bulk = f.bulk;
    const int g = f.g;
    std::string s;
    char line[1024];
    s += kPrelude;
    s += "#include \"tile_kernel.cuh\"\n";
    s += "struct Spec {\n";
    snprintf(line, sizeof line,
             "  static constexpr int n_fir = %d, main_start = %d, reduce = %d;\n"
             "  static constexpr int temps4 = %d, n_tmp = %d;\n"
             "  static constexpr bool tmp_regs = %s;\n",
             P.n_fir, P.main_start, P.reduce, f.temps4, f.n_tmp, f.tmp_regs ? "true" : "false");
    s += line;
    s += "  static constexpr tilek::FirC fir[] = {";
    if (P.n_fir == 0) s += "{0, 0, 0, 0}";
    for (int f = 0; f < P.n_fir; f++) {
        snprintf(line, sizeof line, "%s{%d, %d, %d, %d}", f ? ", " : "", P.fir[f].start,
                 P.fir[f].taps, P.fir[f].head, P.fir[f].tile4);
        s += line;
    }
    s += "};\n  static constexpr tilek::Insn code[] = {\n";
    for (int pc = 0; pc < P.n_code; pc++) {
        const tilek::Insn& in = P.code[pc];
        snprintf(line, sizeof line, "    {%u, %u, %u, %u, %u, 0.0f, 0u},\n", (unsigned)in.op,
                 (unsigned)in.flags, (unsigned)in.a, (unsigned)in.b, (unsigned)in.d);
        s += line;
    }
    s += "  };\n};\n";
    snprintf(line, sizeof line,
             "extern \"C\" __global__ void __launch_bounds__(%d, %d)\n"
             "k_tile_spec(const __grid_constant__ tilek::Program P, float* __restrict__ out,\n"
             "            int64_t n, int64_t halo, bool vec, bool in_vec, int32_t hs,\n"
             "            int32_t stages4, int32_t nst, uint32_t* wd,\n"
             "            int64_t* __restrict__ out_idx, int64_t idx_base) {\n",
             tilek::kThreads, g == tilek::kG ? 3 : 2);
    s += line;
    snprintf(line, sizeof line,
             "  tilek::tile_body<%s, %d, Spec>(P, out, n, halo, vec, in_vec, hs, stages4, nst, wd,\n"
             "                                 out_idx, idx_base);\n}\n",
             bulk ? "true" : "false", g);
    s += line;
    return s;
}

int get(const tilek::Program& P, const Form& f, int dyn_max, CUfunction* out) {
    return get_kernel(spec_source(P, f), "k_tile_spec", nullptr, dyn_max, out);
}

// A streaming reduction's specialised kernel: k_red_direct<kind,
// StaticChain<Steps>> with the chain's steps as constants (the factors stay
// in the parameter block).
std::string chain_source(int kind, const tilek::Chain& ch, std::string* expr_out) {
    std::string src = kPrelude;
    src += "#include \"tile_kernel.cuh\"\nstruct Steps {\n  static constexpr int n = " +
           std::to_string(ch.n) + ";\n  static constexpr int op[] = {";
    for (int i = 0; i < std::max(ch.n, 1); i++)
        src += (i ? ", " : "") + std::to_string(i < ch.n ? ch.op[i] : 0);
    src += "};\n};\n";
    const std::string expr =
        "tilek::k_red_direct<" + std::to_string(kind) + ", tilek::StaticChain<Steps>>";
    src += "template __global__ void " + expr +
           "(const float* __restrict__, int64_t, int64_t, const tilek::Chain, float* "
           "__restrict__, int64_t* __restrict__, int64_t, int64_t);\n";
    *expr_out = expr;
    return src;
}

int get_chain(int kind, const tilek::Chain& ch, CUfunction* out) {
    std::string expr;
    const std::string src = chain_source(kind, ch, &expr);
    return get_kernel(src, nullptr, expr.c_str(), 0, out);
}

int compile_chain_only(int kind, const tilek::Chain& ch) {
    std::call_once(g_rtc_once, open_nvrtc);
    if (!g_rtc.ok) return sg::fail(SIMTGO_EDEVICE, "tile: %s", g_rtc.why.c_str());
    std::string expr;
    const std::string src = chain_source(kind, ch, &expr), id = identity(src);
    Compiled c;
    if (disk_read(id, &c)) {
        g_disk_hits.fetch_add(1);
        return 0;
    }
    if (int rc = compile_source(src, nullptr, expr.c_str(), &c)) return rc;
    g_compiled.fetch_add(1);
    disk_write(id, c);
    return 0;
}

bool available() {
    if (mode() == 0) return false;
    std::call_once(g_rtc_once, open_nvrtc);
    std::call_once(g_drv_once, open_driver);
    // Mode 2 reports true so that get() fails with the reason.
    return mode() == 2 || (g_rtc.ok && g_drv.ok);
}

int compile_only(const tilek::Program& P, const Form& f) {
    std::call_once(g_rtc_once, open_nvrtc);
    if (!g_rtc.ok) return sg::fail(SIMTGO_EDEVICE, "tile: %s", g_rtc.why.c_str());
    const std::string src = spec_source(P, f), id = identity(src);
    Compiled c;
    if (disk_read(id, &c)) {
        g_disk_hits.fetch_add(1);
        return 0;
    }
    if (int rc = compile_source(src, "k_tile_spec", nullptr, &c)) return rc;
    g_compiled.fetch_add(1);
    disk_write(id, c);
    return 0;
}

int occupancy(CUfunction fn, size_t smem, int* blocks) {
    return drv_status(g_drv.occupancy(blocks, fn, tilek::kThreads, smem),
                      "cuOccupancyMaxActiveBlocksPerMultiprocessor(tile)");
}

int launch(CUfunction fn, int blocks, size_t smem, cudaStream_t s, void** args) {
    g_launches.fetch_add(1);
    return drv_status(g_drv.launch(fn, blocks, 1, 1, tilek::kThreads, 1, 1, (unsigned)smem,
                                   (CUstream)s, args, nullptr),
                      "cuLaunchKernel(tile)");
}

}  // namespace tilejit

namespace sg {
// Unloads every specialised kernel's module (simtgo_shutdown), each with its
// device current; later launches compile or load them again.
int tile_jit_release() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_cache.empty()) return 0;
    int prev = 0, rc = 0;
    cudaGetDevice(&prev);
    for (auto& kv : g_cache) {
        int r = cuda_status(cudaSetDevice(kv.second.dev), "cudaSetDevice");
        if (!r && g_drv.unload) r = drv_status(g_drv.unload(kv.second.mod), "cuModuleUnload");
        if (r && !rc) rc = r;
    }
    g_cache.clear();
    cudaSetDevice(prev);
    return rc;
}
}  // namespace sg

extern "C" {

int simtgo_tile_set_jit(int32_t m) {
    sg::clear_error();
    if (m < 0 || m > 2)
        return sg::fail(SIMTGO_EARG, "tile: JIT mode %d is not 0 (off), 1 (on) or 2 (required)",
                        (int)m);
    g_mode.store(m);
    return 0;
}

int simtgo_tile_jit_info(int32_t* m, int32_t* available, int64_t* compiled, int64_t* launches,
                         int64_t* cache_hits) {
    sg::clear_error();
    std::call_once(g_rtc_once, open_nvrtc);
    if (m) *m = mode();
    if (available) *available = g_rtc.ok ? 1 : 0;
    if (compiled) *compiled = g_compiled.load();
    if (launches) *launches = g_launches.load();
    if (cache_hits) *cache_hits = g_disk_hits.load();
    return 0;
}

}  // extern "C"
