// ref_glsl_shim.h -- lets the reference's GLSL compute shaders compile as
// C++ so that the oracle can be checked against the reference's own source.
//
// TEST INFRASTRUCTURE ONLY (oracle/).  ref_glsl.mk strips the #version /
// #extension lines and rewrites each storage-buffer block
//     layout(binding = N) readonly buffer B { T name[]; };
// into GLSL_SSBO(N, T, name); everything else in the shader is compiled as
// written, inside its own namespace, by the definitions below.  Invocations
// of a workgroup run as OpenMP threads when the shader uses barrier(), else
// one after another.
#pragma once

#include <cmath>
#include <cstdint>
#include <omp.h>

typedef unsigned int uint;

struct glsl_uvec3 {
    uint x, y, z;
};

struct uvec4 {
    uint x, y, z, w;
    uvec4() : x(0), y(0), z(0), w(0) {}
    explicit uvec4(uint v) : x(v), y(v), z(v), w(v) {}
    uvec4(uint a, uint b, uint c, uint d) : x(a), y(b), z(c), w(d) {}
    uvec4 &operator+=(const uvec4 &o) {
        x += o.x;
        y += o.y;
        z += o.z;
        w += o.w;
        return *this;
    }
};

// invocation / workgroup ids of the invocation being run
extern thread_local uint glsl_lid;
extern uint glsl_wgid;
extern uint glsl_local_size;

#define layout(...)
#define in
#define uniform struct
#define shared static
#define barrier() _Pragma("omp barrier")
#define GLSL_SSBO(binding, T, name) static T *name
#define gl_LocalInvocationID (glsl_uvec3{glsl_lid, 0u, 0u})
#define gl_WorkGroupID (glsl_uvec3{glsl_wgid, 0u, 0u})
#define gl_GlobalInvocationID (glsl_uvec3{glsl_wgid * glsl_local_size + glsl_lid, 0u, 0u})

// GLSL built-ins used by the shaders, declared inside each shader's namespace
// so that they hide the C library's double versions.
#define GLSL_BUILTINS                                                                        \
    static inline float exp(float v) { return std::exp(v); }                                 \
    static inline float max(float a, float b) { return (a < b) ? b : a; }
