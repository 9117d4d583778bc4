// glsl_cpu.hpp — just enough GLSL (450, compute) semantics to compile AIHost's attention
// shaders (and the weight dequantisation / MatMulWeights shaders beside them) as C++ and run
// them on the CPU. TEST INFRASTRUCTURE ONLY (oracle pinning).
//
// Each shader becomes its own namespace. Invocations of one workgroup run as threads when the
// shader calls barrier(), or one after another when it does not; workgroups run one at a
// time, so `shared` arrays are plain namespace-scope arrays. Built-ins used by the attention
// shaders: max, exp, pow, cos, sin (float), uint, uvec3, gl_* invocation ids, barrier().
// No <cmath>/<algorithm> is included into the shader translation unit, so these float-only
// overloads are the only candidates and fp32 evaluation order is the shader's own.
#pragma once
#include <cstdint>
#include <cstring>

extern "C" {
float expf(float);
float powf(float, float);
float cosf(float);
float sinf(float);
float sqrtf(float);
}

namespace glsl {
typedef unsigned int uint;
struct uvec3 {
  uint x, y, z;
};

extern thread_local uvec3 gl_LocalInvocationID;
extern thread_local uvec3 gl_GlobalInvocationID;
extern thread_local uvec3 gl_WorkGroupID;
void barrier();

// GLSL max(x, y): y if x < y, else x.
inline float max(float x, float y) { return x < y ? y : x; }
inline float min(float x, float y) { return y < x ? y : x; }
inline float exp(float x) { return expf(x); }
inline float pow(float x, float y) { return powf(x, y); }
inline float cos(float x) { return cosf(x); }
inline float sin(float x) { return sinf(x); }
inline float sqrt(float x) { return sqrtf(x); }
// bit reinterpretation (used by the dequantisation shaders' f16tof32)
inline float uintBitsToFloat(uint u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Runs `main_fn` for every invocation of a gx*gy*gz dispatch of workgroups of size `local`.
void dispatch(void (*main_fn)(), uvec3 local, uvec3 groups, bool uses_barrier);
}  // namespace glsl
