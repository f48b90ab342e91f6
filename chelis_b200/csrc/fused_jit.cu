// fused_jit.cu -- FusedElem elementwise groups compiled per chain at run time.
//
// The reference's GPU lane JIT-compiles one kernel string per fused chain
// (crates/chelis-backend-hip/src/kernels.rs fused_elementwise :2391, built
// with hiprtc on every call, runtime/chelis_hip_runtime.h:409-453).  Here the
// chain's steps become straight-line CUDA in one kernel, compiled once with
// NVRTC for sm_100a and kept in a per-device cache keyed by the kernel text
// (dtype, rank, which inputs run along the innermost axis, the steps): shapes
// and strides are kernel arguments, so every tensor size of a given chain
// shares one compiled kernel.  The interpreter in fused.cu stays the path for
// groups this form does not cover (an innermost extent that is not a whole
// number of 16-byte vectors, an input that is neither unit-stride nor
// broadcast along the innermost axis, misaligned bases) and when NVRTC is
// absent.
//
// Layout: a thread takes one 16-byte vector of the output (4 f32 / 2 f64
// consecutive elements of one innermost row); every input with unit
// innermost stride is read as the matching aligned vector, a broadcast input
// (innermost stride 0) as one element.  Element offsets come from the flat
// index by the division-by-invariant-integer decode of fused.cu.
//
// Step semantics are those of fused.cu apply_light / apply_heavy, written
// out per opcode below: IEEE + - * / and sqrt through the _rn intrinsics (no
// contraction), the canonical quiet NaN after every step but MaxElem /
// MinElem, CUDA's libm for the transcendental steps, pow's signaling-NaN rule.
// The kernel is compiled with the library's own floating-point flags, so the
// JIT and the interpreter give the same bits (tested for every opcode).
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "common.cuh"
#include "_gen/crmath_embed.inc"

namespace chelis {
int rows_mode();

namespace fusedjit {

constexpr int THREADS = 256;

// Kernel argument block; the generated source declares the same struct.
struct Args {
    const void *in[fused::MAX_INPUTS];
    void *out;
    long long stride[fused::MAX_INPUTS][fused::MAX_RANK];
    long long shape[fused::MAX_RANK];
    unsigned div_mul[fused::MAX_RANK];
    unsigned div_shr[fused::MAX_RANK];
    long long nvec;
    long long len;
};

const char *kPrelude = R"SRC(
#include "crmath.cuh"
struct Args {
    const void *in[8];
    void *out;
    long long stride[8][6];
    long long shape[6];
    unsigned div_mul[6];
    unsigned div_shr[6];
    long long nvec;
    long long len;
};
__device__ __forceinline__ float cn(float x) { return isnan(x) ? __int_as_float(0x7fc00000) : x; }
__device__ __forceinline__ double cn(double x) { return isnan(x) ? __longlong_as_double(0x7ff8000000000000ll) : x; }
__device__ __forceinline__ bool snan(float x) { return isnan(x) && !(__float_as_uint(x) & 0x00400000u); }
__device__ __forceinline__ bool snan(double x) {
    return isnan(x) && !(static_cast<unsigned long long>(__double_as_longlong(x)) & 0x0008000000000000ull);
}
__device__ __forceinline__ float pw(float x, float y) { return (snan(x) || snan(y)) ? cn(x + y) : cn(powf(x, y)); }
__device__ __forceinline__ double pw(double x, double y) { return (snan(x) || snan(y)) ? cn(x + y) : cn(pow(x, y)); }
template <typename T> __device__ __forceinline__ T mx(T x, T y) { return (isnan(x) || (!isnan(y) && x >= y)) ? x : y; }
template <typename T> __device__ __forceinline__ T mn(T x, T y) { return (isnan(x) || (!isnan(y) && x <= y)) ? x : y; }
)SRC";

// f32 exp / log steps through the correctly rounded functions of crmath.cuh
// (the EXACT rows mode: the C lane's CORE-MATH results bit for bit) rather
// than CUDA's expf / logf; set by the entry that generates the source.
thread_local bool t_correctly_rounded = false;

// One step's expression over operands `a` (and `b`), in the dtype's spelling.
std::string step_expr(int op, bool f32, const std::string &a, const std::string &b) {
    auto fn = [&](const char *f, const char *d) { return std::string(f32 ? f : d); };
    auto un = [&](const char *f, const char *d) { return "cn(" + fn(f, d) + "(" + a + "))"; };
    if (f32 && t_correctly_rounded) {
        if (op == CHELIS_FUSED_EXP) return "cn(chelis::crmath::expf_cr(" + a + "))";
        if (op == CHELIS_FUSED_LOG) return "cn(chelis::crmath::logf_cr(" + a + "))";
    }
    switch (op) {
        case CHELIS_FUSED_ADD: return "cn(" + fn("__fadd_rn", "__dadd_rn") + "(" + a + ", " + b + "))";
        case CHELIS_FUSED_SUB: return "cn(" + fn("__fsub_rn", "__dsub_rn") + "(" + a + ", " + b + "))";
        case CHELIS_FUSED_MUL: return "cn(" + fn("__fmul_rn", "__dmul_rn") + "(" + a + ", " + b + "))";
        case CHELIS_FUSED_DIV: return "cn(" + fn("__fdiv_rn", "__ddiv_rn") + "(" + a + ", " + b + "))";
        case CHELIS_FUSED_POW: return "pw(" + a + ", " + b + ")";
        case CHELIS_FUSED_FLOOR_DIV:
            return "cn(" + fn("floorf", "floor") + "(" + fn("__fdiv_rn", "__ddiv_rn") + "(" + a + ", " + b + ")))";
        case CHELIS_FUSED_MAX_ELEM: return "mx(" + a + ", " + b + ")";
        case CHELIS_FUSED_MIN_ELEM: return "mn(" + a + ", " + b + ")";
        case CHELIS_FUSED_NEG: return "cn(-(" + a + "))";
        case CHELIS_FUSED_RECIP:
            return "cn(" + fn("__fdiv_rn(1.0f, ", "__ddiv_rn(1.0, ") + a + "))";
        case CHELIS_FUSED_EXP: return un("expf", "exp");
        case CHELIS_FUSED_LOG: return un("logf", "log");
        case CHELIS_FUSED_SIN: return un("sinf", "sin");
        case CHELIS_FUSED_SQRT: return un("__fsqrt_rn", "__dsqrt_rn");
        case CHELIS_FUSED_COS: return un("cosf", "cos");
        case CHELIS_FUSED_TAN: return un("tanf", "tan");
        case CHELIS_FUSED_ATAN: return un("atanf", "atan");
        case CHELIS_FUSED_TANH: return un("tanhf", "tanh");
        case CHELIS_FUSED_ERF: return un("erff", "erf");
        case CHELIS_FUSED_ERFC: return un("erfcf", "erfc");
        case CHELIS_FUSED_ABS: return un("fabsf", "fabs");
        case CHELIS_FUSED_FLOOR: return un("floorf", "floor");
        case CHELIS_FUSED_CEIL: return un("ceilf", "ceil");
        case CHELIS_FUSED_ROUND: return un("rintf", "rint");
        default: return "";
    }
}

// Code that evaluates the chain on the V consecutive elements starting at
// flat index `first` (an expression of type long long): their offsets in
// every input, the loads (unit-stride inputs as one vector, broadcast ones as
// one element) and the steps, leaving element e's result in s<last>_<e>.
// Empty when a step has no spelling here.
std::string vector_body(bool f32, const chelis_fused_step *steps, int n_steps, int n_inputs,
                        int rank, uint32_t unit_inner, bool i32, const std::string &first) {
    const int V = f32 ? 4 : 2;
    const std::string T = f32 ? "float" : "double";
    const std::string VT = f32 ? "float4" : "double2";
    const char *lanes[4] = {"x", "y", "z", "w"};
    std::string s;
    if (i32) {
        s += "    unsigned rem = (unsigned)(" + first + ");\n";
        for (int k = 0; k < n_inputs; ++k) s += "    int o" + std::to_string(k) + " = 0;\n";
        for (int d = rank - 1; d >= 0; --d) {
            const std::string D = std::to_string(d);
            if (d > 0) {
                s += "    { const unsigned qd = a.div_mul[" + D + "] ? (__umulhi(rem, a.div_mul[" + D +
                     "]) >> a.div_shr[" + D + "]) : rem;\n";
                s += "      const int c = (int)(rem - qd * (unsigned)a.shape[" + D + "]); rem = qd;\n";
            } else {
                s += "    { const int c = (int)rem;\n";
            }
            for (int k = 0; k < n_inputs; ++k)
                s += "      o" + std::to_string(k) + " += c * (int)a.stride[" + std::to_string(k) + "][" + D + "];\n";
            s += "    }\n";
        }
    } else {
        s += "    long long rem = " + first + ";\n";
        for (int k = 0; k < n_inputs; ++k) s += "    long long o" + std::to_string(k) + " = 0;\n";
        for (int d = rank - 1; d >= 0; --d) {
            const std::string D = std::to_string(d);
            s += "    { long long c = rem;";
            if (d > 0) s += " c = rem % a.shape[" + D + "]; rem /= a.shape[" + D + "];";
            s += "\n";
            for (int k = 0; k < n_inputs; ++k)
                s += "      o" + std::to_string(k) + " += c * a.stride[" + std::to_string(k) + "][" + D + "];\n";
            s += "    }\n";
        }
    }
    for (int k = 0; k < n_inputs; ++k) {
        const std::string K = std::to_string(k);
        if ((unit_inner >> k) & 1) {
            s += "    const " + VT + " v" + K + " = __ldg(reinterpret_cast<const " + VT +
                 " *>(static_cast<const " + T + " *>(a.in[" + K + "]) + o" + K + "));\n";
        } else {
            s += "    const " + T + " b" + K + " = __ldg(static_cast<const " + T + " *>(a.in[" + K +
                 "]) + o" + K + ");\n";
        }
    }
    for (int e = 0; e < V; ++e) {
        const std::string E = std::to_string(e);
        auto operand = [&](int32_t v) -> std::string {
            if (v >= 0) return ((unit_inner >> v) & 1) ? "v" + std::to_string(v) + "." + lanes[e]
                                                       : "b" + std::to_string(v);
            return "s" + std::to_string(-1 - v) + "_" + E;
        };
        for (int j = 0; j < n_steps; ++j) {
            const int op = steps[j].op;
            const bool binary = op <= CHELIS_FUSED_MIN_ELEM;
            const std::string ex = step_expr(op, f32, operand(steps[j].a), binary ? operand(steps[j].b) : "");
            if (ex.empty()) return "";
            s += "    const " + T + " s" + std::to_string(j) + "_" + E + " = " + ex + ";\n";
        }
    }
    return s;
}

// Elementwise kernel: thread q writes output vector q.
std::string kernel_source(bool f32, const chelis_fused_step *steps, int n_steps, int n_inputs,
                          int rank, uint32_t unit_inner, bool i32) {
    const int V = f32 ? 4 : 2;
    const std::string T = f32 ? "float" : "double";
    const std::string VT = f32 ? "float4" : "double2";
    const std::string body = vector_body(f32, steps, n_steps, n_inputs, rank, unit_inner, i32,
                                         "q * " + std::to_string(V));
    if (body.empty()) return "";
    std::string s = kPrelude;
    s += "extern \"C\" __global__ void __launch_bounds__(256) chelis_fused_jit(Args a) {\n";
    s += "  const long long step = (long long)gridDim.x * 256;\n";
    s += "  for (long long q = (long long)blockIdx.x * 256 + threadIdx.x; q < a.nvec; q += step) {\n";
    s += body;
    const std::string last = "s" + std::to_string(n_steps - 1) + "_";
    s += "    reinterpret_cast<" + VT + " *>(static_cast<" + T + " *>(a.out))[q] = make_" + VT + "(";
    for (int e = 0; e < V; ++e) s += (e ? ", " : "") + last + std::to_string(e);
    s += ");\n  }\n}\n";
    return s;
}

// Reduction over the last axis (length a.len, a multiple of 32 V): one warp
// per output w (a.nvec outputs), the leaves of row w at flat indices
// [w * len, (w + 1) * len).  A pass covers 32 V consecutive leaves, lane l
// the aligned group [l V, l V + V): its pair tree, then the warp butterfly
// (adjacent lanes first), give the pass's aligned subtree, pushed onto the
// carry tree (emit.rs emit_carry_tree_push :8129); the carry tree's total is
// the canonical adjacent-pair tree over the row, canonicalised once.  Max
// keeps per lane the maximum and the last index holding it (NaN anywhere
// gives the canonical NaN); lanes merge by value, later index on ties.  The
// same trees, in the same order, as fused.cu reduce_last_kernel.
std::string reduce_source(bool f32, const chelis_fused_step *steps, int n_steps, int n_inputs,
                          int rank, uint32_t unit_inner, bool i32, bool sum) {
    const int V = f32 ? 4 : 2;
    const int PASS = 32 * V;  // leaves one warp covers per pass: a complete subtree
    constexpr int G = 4;      // passes loaded together: G passes from an aligned start are a subtree too
    constexpr int LOG_G = 2;  // (eight measured slower than four: register pressure)
    const std::string T = f32 ? "float" : "double";
    const std::string add = f32 ? "__fadd_rn" : "__dadd_rn";
    const std::string last = "s" + std::to_string(n_steps - 1) + "_";
    auto body_at = [&](const std::string &offset) {
        return vector_body(f32, steps, n_steps, n_inputs, rank, unit_inner, i32,
                           "w * a.len + c0 + " + offset + " + lane * " + std::to_string(V));
    };
    if (body_at("0").empty()) return "";
    // the lane's V leaves as their subtree (sum), or the in-order max update
    auto lane_sum = [&]() {
        if (V == 4)
            return add + "(" + add + "(" + last + "0, " + last + "1), " + add + "(" + last + "2, " + last + "3))";
        return add + "(" + last + "0, " + last + "1)";
    };
    auto max_update = [&](const std::string &offset) {
        std::string u;
        for (int e = 0; e < V; ++e) {
            const std::string v = last + std::to_string(e);
            u += "    if (isnan(" + v + ")) nan = true; else if (!(best > " + v + ")) { best = " + v +
                 "; at = c0 + " + offset + " + lane * " + std::to_string(V) + " + " + std::to_string(e) + "; }\n";
        }
        return u;
    };
    std::string s = kPrelude;
    s += "extern \"C\" __global__ void __launch_bounds__(256) chelis_fused_jit(Args a) {\n";
    s += "  const int lane = threadIdx.x & 31;\n";
    s += "  const long long warps = (long long)gridDim.x * 8;\n";
    s += "  for (long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); w < a.nvec; w += warps) {\n";
    if (sum) {
        s += "  " + T + " level[48]; long long count = 0;\n";
    } else {
        s += "  " + T + " best = " + (f32 ? std::string("__int_as_float(0xff800000)")
                                         : std::string("__longlong_as_double(0xfff0000000000000ll)")) +
             "; long long at = -1; bool nan = false;\n";
    }
    s += "  long long c0 = 0;\n";
    // groups of G passes: every load of the group is issued before the
    // reductions, so a warp keeps G vectors per lane in flight
    s += "  for (; c0 + " + std::to_string(G * PASS) + " <= a.len; c0 += " + std::to_string(G * PASS) + ") {\n";
    if (sum) s += "    " + T + " tg[" + std::to_string(G) + "];\n";
    for (int u = 0; u < G; ++u) {
        const std::string off = std::to_string(u * PASS);
        s += "    {\n" + body_at(off);
        if (sum) s += "    tg[" + std::to_string(u) + "] = " + lane_sum() + ";\n";
        else s += max_update(off);
        s += "    }\n";
    }
    if (sum) {
        s += "    for (int off = 1; off < 32; off <<= 1) {\n";
        s += "      #pragma unroll\n";
        s += "      for (int u = 0; u < " + std::to_string(G) + "; ++u) tg[u] = " + add +
             "(tg[u], __shfl_xor_sync(0xffffffffu, tg[u], off));\n";
        s += "    }\n";
        // the G pass subtrees pair up level by level into the group's subtree
        for (int h = 1; h < G; h <<= 1)
            for (int u = 0; u < G; u += 2 * h)
                s += "    tg[" + std::to_string(u) + "] = " + add + "(tg[" + std::to_string(u) + "], tg[" +
                     std::to_string(u + h) + "]);\n";
        s += "    " + T + " t = tg[0];\n";
        // it enters the carry tree at depth log2(G) (count is a multiple of G here)
        s += "    { int depth = " + std::to_string(LOG_G) + "; for (long long pending = count >> " +
             std::to_string(LOG_G) + "; pending & 1; pending >>= 1, ++depth) t = " + add +
             "(level[depth], t); level[depth] = t; count += " + std::to_string(G) + "; }\n";
    }
    s += "  }\n";
    // the remaining passes, one at a time
    s += "  for (; c0 < a.len; c0 += " + std::to_string(PASS) + ") {\n";
    s += body_at("0");
    if (sum) {
        s += "    " + T + " t = " + lane_sum() + ";\n";
        s += "    for (int off = 1; off < 32; off <<= 1) t = " + add + "(t, __shfl_xor_sync(0xffffffffu, t, off));\n";
        s += "    { int depth = 0; for (long long pending = count++; pending & 1; pending >>= 1, ++depth) t = " +
             add + "(level[depth], t); level[depth] = t; }\n";
    } else {
        s += max_update("0");
    }
    s += "  }\n";
    if (sum) {
        s += "  " + T + " total = 0; bool found = false; int depth = 0;\n";
        s += "  for (long long remaining = count; remaining; remaining >>= 1, ++depth)\n";
        s += "    if (remaining & 1) { total = found ? " + add + "(level[depth], total) : level[depth]; found = true; }\n";
        s += "  if (lane == 0) static_cast<" + T + " *>(a.out)[w] = cn(found ? total : (" + T + ")0);\n";
    } else {
        s += "  nan = __any_sync(0xffffffffu, nan);\n";
        s += "  for (int off = 16; off > 0; off >>= 1) {\n";
        s += "    const " + T + " ob = __shfl_xor_sync(0xffffffffu, best, off);\n";
        s += "    const long long oa = __shfl_xor_sync(0xffffffffu, at, off);\n";
        s += "    if (ob > best || (ob == best && oa > at)) { best = ob; at = oa; }\n";
        s += "  }\n";
        s += "  if (lane == 0) static_cast<" + T + " *>(a.out)[w] = nan ? " +
             (f32 ? std::string("__int_as_float(0x7fc00000)") : std::string("__longlong_as_double(0x7ff8000000000000ll)")) +
             " : best;\n";
    }
    s += "  }\n}\n";
    return s;
}

// ---------------------------------------------------------------------------
// NVRTC (opened at run time: the library links no NVRTC) and the cache
// ---------------------------------------------------------------------------
struct Nvrtc {
    decltype(&nvrtcCreateProgram) create = nullptr;
    decltype(&nvrtcCompileProgram) compile = nullptr;
    decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
    decltype(&nvrtcGetProgramLog) log = nullptr;
    decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
    decltype(&nvrtcGetCUBIN) cubin = nullptr;
    decltype(&nvrtcDestroyProgram) destroy = nullptr;
    bool ok = false;
};

const Nvrtc &nvrtc() {
    static Nvrtc n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnvrtc.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        n.create = reinterpret_cast<decltype(n.create)>(dlsym(h, "nvrtcCreateProgram"));
        n.compile = reinterpret_cast<decltype(n.compile)>(dlsym(h, "nvrtcCompileProgram"));
        n.log_size = reinterpret_cast<decltype(n.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
        n.log = reinterpret_cast<decltype(n.log)>(dlsym(h, "nvrtcGetProgramLog"));
        n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
        n.cubin = reinterpret_cast<decltype(n.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
        n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
        n.ok = n.create && n.compile && n.log_size && n.log && n.cubin_size && n.cubin && n.destroy;
    });
    return n;
}

// Driver entry points through the runtime (the library links no libcuda, so
// it loads on hosts without a driver).
struct Driver {
    decltype(&cuModuleLoadData) load = nullptr;
    decltype(&cuModuleGetFunction) get = nullptr;
    decltype(&cuLaunchKernel) launch = nullptr;
    decltype(&cuModuleUnload) unload = nullptr;
    bool ok = false;
};

const Driver &driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto entry = [](const char *name) -> void * {
            void *ptr = nullptr;
            cudaDriverEntryPointQueryResult q{};
            if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
                q != cudaDriverEntryPointSuccess)
                return nullptr;
            return ptr;
        };
        d.load = reinterpret_cast<decltype(d.load)>(entry("cuModuleLoadData"));
        d.get = reinterpret_cast<decltype(d.get)>(entry("cuModuleGetFunction"));
        d.launch = reinterpret_cast<decltype(d.launch)>(entry("cuLaunchKernel"));
        d.unload = reinterpret_cast<decltype(d.unload)>(entry("cuModuleUnload"));
        d.ok = d.load && d.get && d.launch && d.unload;
    });
    return d;
}

std::mutex g_mu;
std::unordered_map<std::string, CUfunction> g_cache;  // key: device id + kernel text
std::vector<std::pair<int, CUmodule>> g_modules;      // (device, module) behind g_cache
std::atomic<int> g_enabled{1};
std::atomic<uint64_t> g_jit_launches{0};
std::atomic<uint64_t> g_compiles{0};

// Compiled kernel for `src` on the current device (compiling it on first use).
int get_kernel(const std::string &src, CUfunction *fn) {
    int dev = 0;
    CHELIS_TRY(current_device_checked(&dev));
    const std::string key = std::to_string(dev) + "\n" + src;
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_cache.find(key);
    if (it != g_cache.end()) {
        *fn = it->second;
        return CHELIS_CUDA_OK;
    }
    const Nvrtc &n = nvrtc();
    if (!n.ok) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "NVRTC is not available");
    nvrtcProgram prog;
    const char *headers[2] = {kEmbed_crmath_tables_cuh, kEmbed_crmath_cuh};
    const char *names[2] = {"crmath_tables.cuh", "crmath.cuh"};
    if (n.create(&prog, src.c_str(), "chelis_fused_jit.cu", 2, headers, names) != NVRTC_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "nvrtcCreateProgram failed");
    const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "-ftz=false", "-prec-div=true",
                          "-prec-sqrt=true", "-default-device"};
    const nvrtcResult cr = n.compile(prog, 6, opts);
    if (cr != NVRTC_SUCCESS) {
        size_t ls = 0;
        n.log_size(prog, &ls);
        std::string log(ls, '\0');
        if (ls) n.log(prog, &log[0]);
        n.destroy(&prog);
        return set_error(CHELIS_CUDA_ERR_CUDA, "fused JIT compile failed: %.400s", log.c_str());
    }
    size_t bytes = 0;
    n.cubin_size(prog, &bytes);
    std::string cubin(bytes, '\0');
    n.cubin(prog, &cubin[0]);
    n.destroy(&prog);
    CHELIS_TRY(check_cuda(cudaFree(nullptr), "cudaFree(0) (context)"));
    const Driver &drv = driver();
    if (!drv.ok) return set_error(CHELIS_CUDA_ERR_CUDA, "driver module entry points unavailable");
    CUmodule mod;
    if (drv.load(&mod, cubin.data()) != CUDA_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "cuModuleLoadData(fused JIT) failed");
    if (drv.get(fn, mod, "chelis_fused_jit") != CUDA_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "cuModuleGetFunction(fused JIT) failed");
    g_cache.emplace(key, *fn);
    g_modules.emplace_back(dev, mod);
    g_compiles++;
    return CHELIS_CUDA_OK;
}

// Inputs that run along the innermost axis with unit stride (bit k set), or
// false when some input is neither unit-stride nor broadcast there, or a
// unit-stride input cannot be read as aligned V-element vectors.
bool unit_inputs(const fused::Program &p, int V, uint32_t *unit) {
    const int64_t inner = p.shape[p.rank - 1];
    *unit = 0;
    for (int k = 0; k < p.n_inputs; ++k) {
        const int64_t st = inner > 1 ? p.stride[k][p.rank - 1] : 0;
        if (st == 1) {
            if (reinterpret_cast<uintptr_t>(p.in[k]) % 16 != 0) return false;
            for (int d = 0; d < p.rank - 1; ++d)
                if (p.shape[d] > 1 && p.stride[k][d] % V != 0) return false;
            *unit |= 1u << k;
        } else if (st != 0) {
            return false;
        }
    }
    return true;
}

void fill_args(Args &a, const fused::Program &p, void *out, bool i32) {
    a = Args{};
    for (int k = 0; k < p.n_inputs; ++k) {
        a.in[k] = p.in[k];
        for (int d = 0; d < p.rank; ++d) a.stride[k][d] = p.stride[k][d];
    }
    a.out = out;
    for (int d = 0; d < p.rank; ++d) {
        a.shape[d] = p.shape[d];
        uint32_t mul = 0, shr = 0;
        if (i32 && p.shape[d] > 1) {  // fused.cu fast_divisor
            int c = 0;
            while ((uint64_t(1) << c) < static_cast<uint64_t>(p.shape[d])) ++c;
            mul = static_cast<uint32_t>(((uint64_t(1) << (31 + c)) + p.shape[d] - 1) / p.shape[d]);
            shr = static_cast<uint32_t>(c - 1);
        }
        a.div_mul[d] = mul;
        a.div_shr[d] = shr;
    }
}

int launch(CUfunction fn, Args &a, int64_t blocks, cudaStream_t s) {
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    void *params[] = {&a};
    if (driver().launch(fn, static_cast<unsigned>(blocks), 1, 1, THREADS, 1, 1, 0, s, params, nullptr) !=
        CUDA_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "cuLaunchKernel(fused JIT) failed");
    g_launches++;
    g_jit_launches++;
    return CHELIS_CUDA_OK;
}

// Runs the chain through a compiled kernel.  Returns -1 (nothing launched)
// when the group is outside this form or JIT is switched off / unavailable,
// so the caller takes the interpreter; otherwise a status.
int try_elementwise(bool f32, const chelis_fused_step *steps, int n_steps, const fused::Program &p,
                    int mode, void *out, cudaStream_t s) {
    if (!g_enabled.load() || !nvrtc().ok || p.rank < 1 || p.total <= 0) return -1;
    t_correctly_rounded = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    const int V = f32 ? 4 : 2;
    uint32_t unit = 0;
    if (p.shape[p.rank - 1] % V != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0 ||
        !unit_inputs(p, V, &unit))
        return -1;
    const bool i32 = mode != fused::STRIDED64 && p.total < (int64_t(1) << 31);
    const std::string src = kernel_source(f32, steps, n_steps, p.n_inputs, p.rank, unit, i32);
    if (src.empty()) return -1;
    CUfunction fn;
    CHELIS_TRY(get_kernel(src, &fn));
    Args a;
    fill_args(a, p, out, i32);
    a.nvec = p.total / V;
    return launch(fn, a, (a.nvec + THREADS - 1) / THREADS, s);
}

// The chain reduced (Sum or Max) along the last axis, when that axis is a
// whole number of 32-lane passes of V-element vectors and there are enough
// outputs to give every SM eight warps (one warp per output; fewer, longer
// rows go to the interpreter, which splits a row into segments); -1 as above.
int try_reduce(bool f32, const chelis_fused_step *steps, int n_steps, const fused::Program &p,
               int mode, int axis, int kind, int64_t outputs, void *out, cudaStream_t s) {
    if (!g_enabled.load() || !nvrtc().ok || p.rank < 1 || axis != p.rank - 1 || outputs < 1) return -1;
    t_correctly_rounded = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    const int V = f32 ? 4 : 2;
    const int64_t len = p.shape[axis];
    const int64_t want = static_cast<int64_t>(sm_count()) * 8;
    uint32_t unit = 0;
    if (len <= 0 || len % (32 * V) != 0 || !unit_inputs(p, V, &unit)) return -1;
    if (outputs < want) {
        // Few, long rows: cut each row into aligned segments of seg leaves
        // (a power-of-two share of the row, a whole number of passes: every
        // segment is a subtree of the canonical tree), reduce the segments
        // one warp each into partials, then the partials of each row, in
        // order, by the same group kind through an identity step (max_elem
        // of a value with itself keeps its bits).
        // (segments enough for 64 warps per SM, as many rows do; far fewer
        // and longer ones leave the warps latency-bound: measured)
        int64_t seg = len;
        while (outputs * (len / seg) < 8 * want && seg % 2 == 0 && (seg / 2) % (32 * V) == 0) seg /= 2;
        if (outputs * (len / seg) < want) return -1;
        const int64_t nseg = len / seg;
        const bool i32 = mode != fused::STRIDED64 && p.total < (int64_t(1) << 31);
        const std::string src = reduce_source(f32, steps, n_steps, p.n_inputs, p.rank, unit, i32,
                                              kind == CHELIS_FUSED_REDUCE_SUM);
        if (src.empty()) return -1;
        CUfunction fn;
        CHELIS_TRY(get_kernel(src, &fn));
        const size_t elem = f32 ? 4 : 8;
        void *part = nullptr;
        CHELIS_TRY(scratch_alloc(&part, static_cast<size_t>(outputs * nseg) * elem, s));
        Args a;
        fill_args(a, p, part, i32);
        a.nvec = outputs * nseg;  // segment w covers flat leaves [w * seg, (w + 1) * seg)
        a.len = seg;
        int st = launch(fn, a, (a.nvec + THREADS / 32 - 1) / (THREADS / 32), s);
        if (st == CHELIS_CUDA_OK) {
            const chelis_fused_step id{CHELIS_FUSED_MAX_ELEM, 0, 0};
            const void *ins[1] = {part};
            const int64_t strides[2] = {nseg, 1};
            const int64_t shape[2] = {outputs, nseg};
            st = chelis_cuda_fused_reduce(f32 ? CHELIS_DTYPE_F32 : CHELIS_DTYPE_F64, &id, 1, ins, strides,
                                          1, shape, 2, 1, kind, out);
        }
        scratch_free(part, s);
        return st;
    }
    const bool i32 = mode != fused::STRIDED64 && p.total < (int64_t(1) << 31);
    const std::string src = reduce_source(f32, steps, n_steps, p.n_inputs, p.rank, unit, i32,
                                          kind == CHELIS_FUSED_REDUCE_SUM);
    if (src.empty()) return -1;
    CUfunction fn;
    CHELIS_TRY(get_kernel(src, &fn));
    Args a;
    fill_args(a, p, out, i32);
    a.nvec = outputs;
    a.len = len;
    return launch(fn, a, (outputs + THREADS / 32 - 1) / (THREADS / 32), s);
}

// Unload every compiled chain kernel (each on its own device) and empty the
// cache; later calls compile again.
int release_all() {
    std::lock_guard<std::mutex> lock(g_mu);
    int st = CHELIS_CUDA_OK, prev = 0;
    cudaGetDevice(&prev);
    const Driver &drv = driver();
    for (auto &dm : g_modules) {
        if (cudaSetDevice(dm.first) != cudaSuccess || !drv.unload || drv.unload(dm.second) != CUDA_SUCCESS)
            st = set_error(CHELIS_CUDA_ERR_CUDA, "cuModuleUnload(fused JIT) failed");
    }
    cudaSetDevice(prev);
    g_modules.clear();
    g_cache.clear();
    return st;
}

}  // namespace fusedjit
}  // namespace chelis

extern "C" int chelis_cuda_set_fused_jit(int enable) {
    if (enable != 0 && enable != 1)
        return chelis::set_error(CHELIS_CUDA_ERR_DOMAIN, "fused JIT mode must be 0 or 1");
    chelis::fusedjit::g_enabled.store(enable);
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_get_fused_jit(void) { return chelis::fusedjit::g_enabled.load(); }

extern "C" int64_t chelis_cuda_fused_jit_launches(void) {
    return static_cast<int64_t>(chelis::fusedjit::g_jit_launches.load());
}
