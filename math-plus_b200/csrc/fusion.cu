// Element-wise fusion: a traced expression of the tensor-compile IR
// (packages/tensor-compile/src/ir.ts:66-72: input / const / unary / binary / cmp / select nodes)
// lowered to ONE CUDA kernel that reads each input element once and writes each output element
// once, with no intermediate buffers. The reference lowers the same IR to one WGSL shader
// (packages/tensor-webgpu/src/fusion-wgsl.ts:303-431) behind WebGpuDevice.fuse / compile
// (facade.ts:137-164); here the lowering emits CUDA C++, NVRTC compiles it for sm_100a at run time
// (resolved with dlopen, like NCCL), and the driver loads the cubin.
//
// The IR arrives as a DAG of instructions {op, a, b, c} (operands are earlier instruction indices,
// an input index or a constant index) so that a caller in any language can pass it through the
// C ABI. Every node is evaluated in f64, exactly as the reference's CPU evaluator does it
// (evalValue, ir.ts:339-383, on JavaScript numbers), with the value formulas of
// unaryValueAndDeriv (ir.ts:96-215) and JavaScript's Math semantics where C's differ (Math.round,
// Math.sign, Math.pow with NaN or ±1 ** ±Infinity, min / max as `l <= r ? l : r`); the result is
// rounded once to f32 on store, as CompiledFn.forward stores into a Float32Array. Multiply-add
// contraction is off, so a*b+c rounds twice like the reference.
//
// Two kernels per expression: a flat one (every input contiguous with the output's shape; each
// thread keeps four elements in flight) and a strided one (NumPy broadcasting through element
// strides aligned to the output shape, up to 6 axes).
#include <dlfcn.h>

#include <cctype>
#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <string>

#include "mpc_internal.h"

struct mpc_fused {
  mpc_device *dev = nullptr;
  int n_inputs = 0;
  CUmodule mod = nullptr;
  int dtypes[16] = {0};
  CUfunction flat = nullptr, flat1 = nullptr, strided = nullptr;
};

namespace mpc {
namespace {

constexpr int kMaxInputs = 16;
constexpr int kMaxRank = 6;
constexpr int kMaxInstr = 1 << 16;

// Mirrors the struct the generated source declares.
struct FusedParams {
  const void *in[kMaxInputs];
  long long n;
  int rank;
  long long shape[kMaxRank];
  long long st[kMaxInputs][kMaxRank];
  float *out;
};

// ---- NVRTC and the driver's module calls, resolved at run time ---------------------------------
typedef int nvrtcResult_t;
typedef void *nvrtcProgram_t;

struct NvrtcApi {
  nvrtcResult_t (*Create)(nvrtcProgram_t *, const char *, const char *, int, const char *const *,
                          const char *const *) = nullptr;
  nvrtcResult_t (*Compile)(nvrtcProgram_t, int, const char *const *) = nullptr;
  nvrtcResult_t (*LogSize)(nvrtcProgram_t, size_t *) = nullptr;
  nvrtcResult_t (*Log)(nvrtcProgram_t, char *) = nullptr;
  nvrtcResult_t (*CubinSize)(nvrtcProgram_t, size_t *) = nullptr;
  nvrtcResult_t (*Cubin)(nvrtcProgram_t, char *) = nullptr;
  nvrtcResult_t (*Destroy)(nvrtcProgram_t *) = nullptr;
  const char *(*ErrorString)(nvrtcResult_t) = nullptr;
  bool ok = false;
  char why[256] = {0};
};

const NvrtcApi &nvrtc() {
  static NvrtcApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("/usr/local/cuda/lib64/libnvrtc.so.12", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "dlopen(libnvrtc.so.12): %s", dlerror());
      return;
    }
    api.Create = reinterpret_cast<decltype(api.Create)>(dlsym(h, "nvrtcCreateProgram"));
    api.Compile = reinterpret_cast<decltype(api.Compile)>(dlsym(h, "nvrtcCompileProgram"));
    api.LogSize = reinterpret_cast<decltype(api.LogSize)>(dlsym(h, "nvrtcGetProgramLogSize"));
    api.Log = reinterpret_cast<decltype(api.Log)>(dlsym(h, "nvrtcGetProgramLog"));
    api.CubinSize = reinterpret_cast<decltype(api.CubinSize)>(dlsym(h, "nvrtcGetCUBINSize"));
    api.Cubin = reinterpret_cast<decltype(api.Cubin)>(dlsym(h, "nvrtcGetCUBIN"));
    api.Destroy = reinterpret_cast<decltype(api.Destroy)>(dlsym(h, "nvrtcDestroyProgram"));
    api.ErrorString = reinterpret_cast<decltype(api.ErrorString)>(dlsym(h, "nvrtcGetErrorString"));
    api.ok = api.Create && api.Compile && api.LogSize && api.Log && api.CubinSize && api.Cubin && api.Destroy &&
             api.ErrorString;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnvrtc.so.12 lacks an expected symbol");
  });
  return api;
}

struct DriverApi {
  CUresult (*LoadData)(CUmodule *, const void *) = nullptr;
  CUresult (*GetFunction)(CUfunction *, CUmodule, const char *) = nullptr;
  CUresult (*Launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                     void **, void **) = nullptr;
  CUresult (*Unload)(CUmodule) = nullptr;
  bool ok = false;
};

const DriverApi &driver() {
  static DriverApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char *name) -> void * {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
      return p;
    };
    api.LoadData = reinterpret_cast<decltype(api.LoadData)>(get("cuModuleLoadData"));
    api.GetFunction = reinterpret_cast<decltype(api.GetFunction)>(get("cuModuleGetFunction"));
    api.Launch = reinterpret_cast<decltype(api.Launch)>(get("cuLaunchKernel"));
    api.Unload = reinterpret_cast<decltype(api.Unload)>(get("cuModuleUnload"));
    api.ok = api.LoadData && api.GetFunction && api.Launch && api.Unload;
  });
  return api;
}

// ---- lowering ----------------------------------------------------------------------------------
// The value formula of each UnaryOp (ir.ts:96-215) as a C++ expression of `x`.
const char *unary_formula(int op) {
  switch (op) {
    case MPC_IR_NEG: return "(-x)";
    case MPC_IR_RELU: return "(x > 0.0 ? x : 0.0)";
    case MPC_IR_SIGMOID: return "(1.0 / (1.0 + exp(-x)))";
    case MPC_IR_GELU: return "(x * normcdf(x))";
    case MPC_IR_GELU_TANH: return "(0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x))))";
    case MPC_IR_EXP: return "exp(x)";
    case MPC_IR_LOG: return "log(x)";
    case MPC_IR_SQRT: return "sqrt(x)";
    case MPC_IR_SIN: return "sin(x)";
    case MPC_IR_COS: return "cos(x)";
    case MPC_IR_TAN: return "tan(x)";
    case MPC_IR_ASIN: return "asin(x)";
    case MPC_IR_ACOS: return "acos(x)";
    case MPC_IR_ATAN: return "atan(x)";
    case MPC_IR_SINH: return "sinh(x)";
    case MPC_IR_COSH: return "cosh(x)";
    case MPC_IR_TANH: return "tanh(x)";
    case MPC_IR_COT: return "(1.0 / tan(x))";
    case MPC_IR_SEC: return "(1.0 / cos(x))";
    case MPC_IR_CSC: return "(1.0 / sin(x))";
    case MPC_IR_ASINH: return "asinh(x)";
    case MPC_IR_ACOSH: return "acosh(x)";
    case MPC_IR_ATANH: return "atanh(x)";
    case MPC_IR_COTH: return "(1.0 / tanh(x))";
    case MPC_IR_SECH: return "(1.0 / cosh(x))";
    case MPC_IR_CSCH: return "(1.0 / sinh(x))";
    case MPC_IR_ACOT: return "atan(1.0 / x)";
    case MPC_IR_ASEC: return "acos(1.0 / x)";
    case MPC_IR_ACSC: return "asin(1.0 / x)";
    case MPC_IR_ACOTH: return "(0.5 * log((x + 1.0) / (x - 1.0)))";
    case MPC_IR_ASECH: return "acosh(1.0 / x)";
    case MPC_IR_ACSCH: return "asinh(1.0 / x)";
    case MPC_IR_ABS: return "fabs(x)";
    case MPC_IR_LOG10: return "log10(x)";
    case MPC_IR_LOG2: return "log2(x)";
    case MPC_IR_CBRT: return "cbrt(x)";
    case MPC_IR_FLOOR: return "floor(x)";
    case MPC_IR_CEIL: return "ceil(x)";
    case MPC_IR_ROUND: return "js_round(x)";
    case MPC_IR_SIGN: return "js_sign(x)";
    case MPC_IR_TRUNC: return "trunc(x)";
    case MPC_IR_EXPM1: return "expm1(x)";
    case MPC_IR_LOG1P: return "log1p(x)";
    case MPC_IR_ERF: return "erf(x)";
    default: return nullptr;
  }
}

const char *binary_formula(int op) {
  switch (op) {
    case MPC_IR_ADD: return "(l + r)";
    case MPC_IR_SUB: return "(l - r)";
    case MPC_IR_MUL: return "(l * r)";
    case MPC_IR_DIV: return "(l / r)";
    case MPC_IR_POW: return "js_pow(l, r)";
    case MPC_IR_ATAN2: return "atan2(l, r)";
    case MPC_IR_HYPOT: return "hypot(l, r)";
    case MPC_IR_MIN: return "(l <= r ? l : r)";
    case MPC_IR_MAX: return "(l >= r ? l : r)";
    case MPC_IR_LT: return "(l < r ? 1.0 : 0.0)";
    case MPC_IR_LE: return "(l <= r ? 1.0 : 0.0)";
    case MPC_IR_GT: return "(l > r ? 1.0 : 0.0)";
    case MPC_IR_GE: return "(l >= r ? 1.0 : 0.0)";
    case MPC_IR_EQ: return "(l == r ? 1.0 : 0.0)";
    case MPC_IR_NE: return "(l != r ? 1.0 : 0.0)";
    default: return nullptr;
  }
}

// Substitutes the operand names into a formula: `x` (unary) or `l` / `r` (binary) as whole words.
std::string substitute(const char *formula, const std::string &x, const std::string &l, const std::string &r) {
  std::string out;
  for (const char *p = formula; *p; ++p) {
    const bool word_start = p == formula || !(isalnum((unsigned char)p[-1]) || p[-1] == '_');
    const bool word_end = !(isalnum((unsigned char)p[1]) || p[1] == '_');
    if (word_start && word_end && (*p == 'x' || *p == 'l' || *p == 'r')) {
      out += *p == 'x' ? x : (*p == 'l' ? l : r);
    } else {
      out += *p;
    }
  }
  return out;
}

const char *kPrelude = R"(typedef long long i64;
struct MpcFusedParams {
  const void *in[16];
  i64 n;
  int rank;
  i64 shape[6];
  i64 st[16][6];
  float *out;
};
__device__ __forceinline__ real ld_f32(const void *p, i64 i) { return (real)((const float *)p)[i]; }
__device__ __forceinline__ real ld_f16(const void *p, i64 i) {
  unsigned short h = ((const unsigned short *)p)[i];
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return (real)f;
}
__device__ __forceinline__ real ld_bf16(const void *p, i64 i) {
  return (real)__uint_as_float(((unsigned int)((const unsigned short *)p)[i]) << 16);
}
__device__ __forceinline__ real h2d(unsigned int h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"((unsigned short)h));
  return (real)f;
}
__device__ __forceinline__ real b2d(unsigned int b) { return (real)__uint_as_float(b << 16); }
__device__ __forceinline__ void ld4_f32(const void *p, i64 q, real (&v)[4]) {
  const float4 t = ((const float4 *)p)[q];
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
__device__ __forceinline__ void ld4_f16(const void *p, i64 q, real (&v)[4]) {
  const uint2 t = ((const uint2 *)p)[q];
  v[0] = h2d(t.x & 0xffffu); v[1] = h2d(t.x >> 16); v[2] = h2d(t.y & 0xffffu); v[3] = h2d(t.y >> 16);
}
__device__ __forceinline__ void ld4_bf16(const void *p, i64 q, real (&v)[4]) {
  const uint2 t = ((const uint2 *)p)[q];
  v[0] = b2d(t.x & 0xffffu); v[1] = b2d(t.x >> 16); v[2] = b2d(t.y & 0xffffu); v[3] = b2d(t.y >> 16);
}
// Math.round: the nearest integer, ties toward +Infinity; -0 for x in [-0.5, -0].
__device__ __forceinline__ double js_round(double x) {
  double f = floor(x);
  double r = (x - f >= 0.5) ? f + 1.0 : f;
  return r == 0.0 ? copysign(0.0, x) : r;
}
__device__ __forceinline__ float js_round(float x) {
  float f = floorf(x);
  float r = (x - f >= 0.5f) ? f + 1.0f : f;
  return r == 0.0f ? copysignf(0.0f, x) : r;
}
// Math.sign: NaN stays NaN, a zero keeps its sign.
__device__ __forceinline__ double js_sign(double x) { return x > 0.0 ? 1.0 : (x < 0.0 ? -1.0 : x); }
__device__ __forceinline__ float js_sign(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : x); }
// Math.pow: NaN for a NaN exponent and for (+-1) ** (+-Infinity), where C's pow gives 1.
__device__ __forceinline__ double js_pow(double l, double r) {
  if (r != r) return __longlong_as_double(0x7ff8000000000000LL);
  if (fabs(l) == 1.0 && isinf(r)) return __longlong_as_double(0x7ff8000000000000LL);
  return pow(l, r);
}
__device__ __forceinline__ float js_pow(float l, float r) {
  if (r != r) return __int_as_float(0x7fc00000);
  if (fabsf(l) == 1.0f && isinf(r)) return __int_as_float(0x7fc00000);
  return powf(l, r);
}
)";

const char *loader_of(int dt) {
  switch (dt) {
    case MPC_F32: return "ld_f32";
    case MPC_F16: return "ld_f16";
    case MPC_BF16: return "ld_bf16";
    default: return nullptr;
  }
}

int validate(const int32_t *code, int32_t n_instr, int32_t n_consts, int32_t n_inputs, const int32_t *dtypes) {
  if (n_inputs < 1 || n_inputs > kMaxInputs)
    return fail(MPC_ERR_INVALID, "fusion: %d inputs (1..%d)", n_inputs, kMaxInputs);
  if (!dtypes) return fail(MPC_ERR_INVALID, "fusion: null dtypes");
  for (int j = 0; j < n_inputs; ++j)
    if (!loader_of(dtypes[j])) return fail(MPC_ERR_INVALID, "fusion: input %d has dtype %d (f32, f16, bf16)", j, dtypes[j]);
  if (!code || n_instr < 1 || n_instr > kMaxInstr)
    return fail(MPC_ERR_INVALID, "fusion: %d instructions (1..%d)", n_instr, kMaxInstr);
  if (n_consts < 0) return fail(MPC_ERR_INVALID, "fusion: negative constant count");
  for (int i = 0; i < n_instr; ++i) {
    const int32_t op = code[4 * i], a = code[4 * i + 1], b = code[4 * i + 2], c = code[4 * i + 3];
    auto ref_ok = [i](int32_t v) { return v >= 0 && v < i; };
    if (op == MPC_IR_INPUT) {
      if (a < 0 || a >= n_inputs)
        return fail(MPC_ERR_INVALID, "fusion: IR references input %d, but numInputs is %d", a, n_inputs);
    } else if (op == MPC_IR_CONST) {
      if (a < 0 || a >= n_consts) return fail(MPC_ERR_INVALID, "fusion: instruction %d: constant %d of %d", i, a, n_consts);
    } else if (unary_formula(op)) {
      if (!ref_ok(a)) return fail(MPC_ERR_INVALID, "fusion: instruction %d: operand %d", i, a);
    } else if (binary_formula(op)) {
      if (!ref_ok(a) || !ref_ok(b)) return fail(MPC_ERR_INVALID, "fusion: instruction %d: operands %d, %d", i, a, b);
    } else if (op == MPC_IR_SELECT) {
      if (!ref_ok(a) || !ref_ok(b) || !ref_ok(c))
        return fail(MPC_ERR_INVALID, "fusion: instruction %d: operands %d, %d, %d", i, a, b, c);
    } else {
      return fail(MPC_ERR_INVALID, "fusion: instruction %d: unknown op %d", i, op);
    }
  }
  return MPC_OK;
}

std::string temp(int i) { return "t" + std::to_string(i); }

// A formula for f32 evaluation: the math functions' float versions and float literals.
std::string to_f32(const std::string &e) {
  static const char *kFns[] = {"exp", "log", "sqrt", "sin", "cos", "tan", "asin", "acos", "atan", "sinh", "cosh",
                               "tanh", "asinh", "acosh", "atanh", "fabs", "log10", "log2", "cbrt", "floor", "ceil",
                               "trunc", "expm1", "log1p", "erf", "normcdf", "atan2", "hypot"};
  std::string out;
  size_t i = 0;
  while (i < e.size()) {
    const char ch = e[i];
    if (isalpha((unsigned char)ch) || ch == '_') {  // an identifier
      size_t j = i;
      while (j < e.size() && (isalnum((unsigned char)e[j]) || e[j] == '_')) ++j;
      std::string id = e.substr(i, j - i);
      if (j < e.size() && e[j] == '(')
        for (const char *f : kFns)
          if (id == f) {
            id += 'f';
            break;
          }
      out += id;
      i = j;
    } else if (isdigit((unsigned char)ch)) {  // a number: decimal literals become float literals
      size_t j = i;
      bool dot = false;
      while (j < e.size() && (isdigit((unsigned char)e[j]) || e[j] == '.')) dot |= e[j++] == '.';
      out += e.substr(i, j - i);
      if (dot) out += 'f';
      i = j;
    } else {
      out += ch;
      ++i;
    }
  }
  return out;
}

// CUDA source for a validated program: an eval function over the inputs' values (f64, or f32 with
// MPC_FUSED_F32) and the kernels around it.
std::string lower(const int32_t *code, int32_t n_instr, const double *consts, int32_t n_inputs,
                  const int32_t *dtypes, bool f32) {
  std::string s = f32 ? "typedef float real;\n" : "typedef double real;\n";
  s += kPrelude;
  s += "__device__ __forceinline__ real mpc_eval(";
  for (int j = 0; j < n_inputs; ++j) s += (j ? ", real x" : "real x") + std::to_string(j);
  s += ") {\n";
  for (int i = 0; i < n_instr; ++i) {
    const int32_t op = code[4 * i], a = code[4 * i + 1], b = code[4 * i + 2], c = code[4 * i + 3];
    std::string e;
    if (op == MPC_IR_INPUT) {
      e = "x" + std::to_string(a);
    } else if (op == MPC_IR_CONST) {
      uint64_t bits;
      memcpy(&bits, &consts[a], sizeof bits);
      char buf[64];
      snprintf(buf, sizeof buf, f32 ? "(float)__longlong_as_double(0x%016" PRIx64 "LL)"
                                     : "__longlong_as_double(0x%016" PRIx64 "LL)", bits);
      e = buf;
    } else if (const char *u = unary_formula(op)) {
      e = substitute(u, temp(a), "", "");
    } else if (const char *f = binary_formula(op)) {
      e = substitute(f, "", temp(a), temp(b));
    } else {  // select: nonzero condition takes `then` (NaN counts as nonzero, as in JavaScript)
      e = "(" + temp(a) + " != 0.0 ? " + temp(b) + " : " + temp(c) + ")";
    }
    if (f32 && op != MPC_IR_CONST) e = to_f32(e);
    s += "  const real " + temp(i) + " = " + e + ";\n";
  }
  s += "  return " + temp(n_instr - 1) + ";\n}\n";

  // per input: a scalar load at element i, a 4-wide load of vector q, and a strided load
  std::string args_flat, args_vec[4], loads_vec, args_strided;
  for (int j = 0; j < n_inputs; ++j) {
    const std::string ld = loader_of(dtypes[j]), js = std::to_string(j);
    args_flat += (j ? ", " : "") + ld + "(p.in[" + js + "], i)";
    loads_vec += "      real v" + js + "[4];\n      " + std::string(dtypes[j] == MPC_F32 ? "ld4_f32" : (dtypes[j] == MPC_F16 ? "ld4_f16" : "ld4_bf16")) +
                 "(p.in[" + js + "], q, v" + js + ");\n";
    for (int u = 0; u < 4; ++u) args_vec[u] += (j ? ", v" : "v") + js + "[" + std::to_string(u) + "]";
    args_strided += (j ? ", " : "") + ld + "(p.in[" + js + "], o[" + js + "] + c * p.st[" + js + "][last])";
  }
  const std::string nin = std::to_string(n_inputs);
  // Contiguous inputs: four elements per thread through 16-byte (f32) or 8-byte (16-bit) loads and
  // a 16-byte store; the last n % 4 elements by block 0.
  s += "extern \"C\" __global__ void __launch_bounds__(256) mpc_fused_flat(const MpcFusedParams p) {\n"
       "  const i64 nv = p.n >> 2;\n"
       "  for (i64 q = (i64)blockIdx.x * 256 + threadIdx.x; q < nv; q += (i64)gridDim.x * 256) {\n" +
       loads_vec +
       "      float4 r;\n"
       "      r.x = (float)(mpc_eval(" + args_vec[0] + "));\n"
       "      r.y = (float)(mpc_eval(" + args_vec[1] + "));\n"
       "      r.z = (float)(mpc_eval(" + args_vec[2] + "));\n"
       "      r.w = (float)(mpc_eval(" + args_vec[3] + "));\n"
       "      ((float4 *)p.out)[q] = r;\n"
       "  }\n"
       "  if (blockIdx.x == 0)\n"
       "    for (i64 i = (nv << 2) + threadIdx.x; i < p.n; i += 256) p.out[i] = (float)(mpc_eval(" + args_flat + "));\n"
       "}\n";
  // Contiguous inputs at any alignment: one element per thread.
  s += "extern \"C\" __global__ void __launch_bounds__(256) mpc_fused_flat1(const MpcFusedParams p) {\n"
       "  for (i64 i = (i64)blockIdx.x * 256 + threadIdx.x; i < p.n; i += (i64)gridDim.x * 256)\n"
       "    p.out[i] = (float)(mpc_eval(" + args_flat + "));\n"
       "}\n";
  // Broadcasting: tiles of 1024 elements along the last axis; a tile's row offsets are decoded once.
  s += "extern \"C\" __global__ void __launch_bounds__(256) mpc_fused_strided(const MpcFusedParams p) {\n"
       "  const int last = p.rank - 1;\n"
       "  const i64 inner = p.shape[last];\n"
       "  const i64 tpr = (inner + 1023) >> 10;\n"
       "  const i64 tiles = (p.n / inner) * tpr;\n"
       "  for (i64 t = blockIdx.x; t < tiles; t += gridDim.x) {\n"
       "    const i64 row = t / tpr, c0 = (t - row * tpr) << 10;\n"
       "    i64 o[" + nin + "];\n"
       "#pragma unroll\n"
       "    for (int j = 0; j < " + nin + "; ++j) o[j] = 0;\n"
       "    i64 rem = row;\n"
       "    for (int k = last - 1; k >= 0; --k) {\n"
       "      const i64 q = rem / p.shape[k], c = rem - q * p.shape[k];\n"
       "      rem = q;\n"
       "#pragma unroll\n"
       "      for (int j = 0; j < " + nin + "; ++j) o[j] += c * p.st[j][k];\n"
       "    }\n"
       "#pragma unroll\n"
       "    for (int u = 0; u < 4; ++u) {\n"
       "      const i64 c = c0 + u * 256 + threadIdx.x;\n"
       "      if (c < inner) p.out[row * inner + c] = (float)(mpc_eval(" + args_strided + "));\n"
       "    }\n"
       "  }\n"
       "}\n";
  return s;
}

// NVRTC compile for sm_100a: the cubin, or an error with the compiler's log.
int compile(const std::string &src, std::string &cubin) {
  const NvrtcApi &nv = nvrtc();
  if (!nv.ok) return fail(MPC_ERR_COMPILE, "fusion needs NVRTC: %s", nv.why);
  nvrtcProgram_t prog = nullptr;
  int r = nv.Create(&prog, src.c_str(), "mpc_fused.cu", 0, nullptr, nullptr);
  if (r) return fail(MPC_ERR_COMPILE, "nvrtcCreateProgram: %s", nv.ErrorString(r));
  const char *opts[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--std=c++17", "-default-device"};
  r = nv.Compile(prog, 4, opts);
  if (r) {
    size_t n = 0;
    nv.LogSize(prog, &n);
    std::string log(n, '\0');
    if (n) nv.Log(prog, &log[0]);
    nv.Destroy(&prog);
    return fail(MPC_ERR_COMPILE, "fusion: NVRTC failed (%s): %.400s", nv.ErrorString(r), log.c_str());
  }
  size_t n = 0;
  nv.CubinSize(prog, &n);
  cubin.assign(n, '\0');
  if (n) nv.Cubin(prog, &cubin[0]);
  nv.Destroy(&prog);
  return n ? MPC_OK : fail(MPC_ERR_COMPILE, "fusion: NVRTC produced no cubin");
}

unsigned grid_for_n(mpc_device *dev, long long n, long long per_block) {
  const long long cap = (long long)dev->prop.multiProcessorCount * 8;
  long long g = (n + per_block - 1) / per_block;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace mpc

using namespace mpc;

extern "C" {

int mpc_fused_lower(const int32_t *code, int32_t n_instr, const double *consts, int32_t n_consts, int32_t n_inputs,
                    const int32_t *dtypes, uint32_t flags, int32_t check_compile, char *buf, size_t cap,
                    size_t *len) {
  int rc = validate(code, n_instr, n_consts, n_inputs, dtypes);
  if (rc) return rc;
  if (flags & ~MPC_FUSED_F32) return fail(MPC_ERR_INVALID, "fusion: unknown flags 0x%x", flags);
  const std::string src = lower(code, n_instr, consts, n_inputs, dtypes, flags & MPC_FUSED_F32);
  if (len) *len = src.size();
  if (buf && cap) {
    const size_t n = src.size() < cap - 1 ? src.size() : cap - 1;
    memcpy(buf, src.data(), n);
    buf[n] = '\0';
  }
  if (check_compile) {
    std::string cubin;
    if ((rc = compile(src, cubin))) return rc;
  }
  return MPC_OK;
}

int mpc_fused_create_ex(mpc_device *dev, const int32_t *code, int32_t n_instr, const double *consts,
                        int32_t n_consts, int32_t n_inputs, const int32_t *dtypes, uint32_t flags, mpc_fused **out) {
  int rc = enter(dev);
  if (rc) return rc;
  if (!out) return fail(MPC_ERR_INVALID, "mpc_fused_create: null output");
  *out = nullptr;
  if ((rc = validate(code, n_instr, n_consts, n_inputs, dtypes))) return rc;
  if (flags & ~MPC_FUSED_F32) return fail(MPC_ERR_INVALID, "fusion: unknown flags 0x%x", flags);
  const DriverApi &drv = driver();
  if (!drv.ok) return fail(MPC_ERR_UNSUPPORTED, "fusion: the driver's module entry points are unavailable");
  std::string cubin;
  if ((rc = compile(lower(code, n_instr, consts, n_inputs, dtypes, flags & MPC_FUSED_F32), cubin))) return rc;
  MPC_CUDA(dev, cudaFree(nullptr));  // the device's primary context is current from here on
  auto *f = new mpc_fused;
  f->dev = dev;
  f->n_inputs = n_inputs;
  CUresult r = drv.LoadData(&f->mod, cubin.data());
  for (int j = 0; j < n_inputs; ++j) f->dtypes[j] = dtypes[j];
  if (r == CUDA_SUCCESS) r = drv.GetFunction(&f->flat, f->mod, "mpc_fused_flat");
  if (r == CUDA_SUCCESS) r = drv.GetFunction(&f->flat1, f->mod, "mpc_fused_flat1");
  if (r == CUDA_SUCCESS) r = drv.GetFunction(&f->strided, f->mod, "mpc_fused_strided");
  if (r != CUDA_SUCCESS) {
    if (f->mod) drv.Unload(f->mod);
    delete f;
    return fail(MPC_ERR_CUDA, "fusion: loading the compiled kernel failed (CUresult %d)", (int)r);
  }
  *out = f;
  return MPC_OK;
}

int mpc_fused_create(mpc_device *dev, const int32_t *code, int32_t n_instr, const double *consts, int32_t n_consts,
                     int32_t n_inputs, const int32_t *dtypes, mpc_fused **out) {
  return mpc_fused_create_ex(dev, code, n_instr, consts, n_consts, n_inputs, dtypes, 0, out);
}

int mpc_fused_run(mpc_fused *f, const void *const *inputs, int32_t rank, const int64_t *shape,
                  const int64_t *strides, float *out, mpc_stream s) {
  if (!f) return fail(MPC_ERR_INVALID, "mpc_fused_run: null kernel");
  mpc_device *dev = f->dev;
  int rc = enter(dev);
  if (rc) return rc;
  if (rank < 0 || rank > kMaxRank) return fail(MPC_ERR_UNSUPPORTED, "mpc_fused_run: rank %d (at most %d)", rank, kMaxRank);
  if (rank > 0 && (!shape || !strides)) return fail(MPC_ERR_INVALID, "mpc_fused_run: null shape / strides");
  long long n = 1;
  for (int k = 0; k < rank; ++k) {
    if (shape[k] < 0) return fail(MPC_ERR_INVALID, "mpc_fused_run: negative extent");
    n *= shape[k];
  }
  if (n == 0) return MPC_OK;
  if (!inputs || !out) return fail(MPC_ERR_INVALID, "mpc_fused_run: null pointer");
  for (int j = 0; j < f->n_inputs; ++j)
    if (!inputs[j]) return fail(MPC_ERR_INVALID, "mpc_fused_run: input %d is null", j);
  // Collapse the axes: drop extents of 1, then merge an axis into the next one where every input
  // steps across the pair as across one axis (the output is contiguous, so it always does).
  FusedParams p{};
  int r = 0;
  for (int k = 0; k < rank; ++k) {
    if (shape[k] == 1) continue;
    if (r > 0) {
      bool merge = true;
      for (int j = 0; j < f->n_inputs && merge; ++j)
        merge = p.st[j][r - 1] == strides[(size_t)j * rank + k] * shape[k];
      if (merge) {
        p.shape[r - 1] *= shape[k];
        for (int j = 0; j < f->n_inputs; ++j) p.st[j][r - 1] = strides[(size_t)j * rank + k];
        continue;
      }
    }
    p.shape[r] = shape[k];
    for (int j = 0; j < f->n_inputs; ++j) p.st[j][r] = strides[(size_t)j * rank + k];
    ++r;
  }
  p.rank = r;
  p.n = n;
  p.out = out;
  bool flat = true, aligned = ((uintptr_t)out % 16) == 0;
  for (int j = 0; j < f->n_inputs; ++j) {
    p.in[j] = inputs[j];
    if (r > 0 && p.st[j][r - 1] != 1) flat = false;
    if (r > 1) flat = false;
    const size_t vec = 4 * dtype_size(f->dtypes[j]);
    if ((uintptr_t)inputs[j] % vec) aligned = false;
  }
  CUfunction fn = flat ? (aligned ? f->flat : f->flat1) : f->strided;
  const char *name = flat ? (aligned ? "mpc_fused_flat" : "mpc_fused_flat1") : "mpc_fused_strided";
  long long units = flat ? (aligned ? (n >> 2) : n) : (n / p.shape[r - 1]) * ((p.shape[r - 1] + 1023) >> 10) * 256;
  const unsigned grid = grid_for_n(dev, units > 0 ? units : 1, 256);
  void *args[] = {&p};
  const CUresult cr = driver().Launch(fn, grid, 1, 1, 256, 1, 1, 0, (CUstream)stream_of(dev, s), args, nullptr);
  if (cr != CUDA_SUCCESS) return fail(MPC_ERR_CUDA, "mpc_fused_run: launch failed (CUresult %d)", (int)cr);
  dev->launches++;
  return check_launch(dev, name);
}

int mpc_fused_destroy(mpc_fused *f) {
  if (!f) return MPC_OK;
  if (f->mod) {
    enter(f->dev);
    driver().Unload(f->mod);
  }
  delete f;
  return MPC_OK;
}

}  // extern "C"
