// ORACLE (test infrastructure only): the Metal Shading Language constructs the
// reference's compute kernels (metal_llm.metal) use, restated as C++ so that
// those kernels compile with g++ where they lie and run on the host
// (oracle/metal_ref.cpp).  Address-space qualifiers and `kernel` vanish,
// `threadgroup` arrays become function statics (one threadgroup runs at a
// time), the Metal scalar and vector types are plain structs, and the math
// functions are the host's single-precision libm calls, so a kernel runs its
// own arithmetic in its own order in IEEE FP32 (the GPU's fast-math
// approximations are not reproduced).
#pragma once

#define kernel
#define device
#define constant const
#define thread
#define threadgroup static

typedef unsigned int uint;
typedef unsigned char uchar;
typedef unsigned short ushort;
typedef _Float16 half;

struct uint2 {
    uint x, y;
    uint2() = default;
    constexpr uint2(uint a, uint b) : x(a), y(b) {}
};
struct uint3 {
    uint x, y, z;
    uint3() = default;
    constexpr uint3(uint a, uint b, uint c) : x(a), y(b), z(c) {}
};

template <class T, class U>
inline T as_type(U u) {
    static_assert(sizeof(T) == sizeof(U), "as_type: sizes differ");
    T t;
    __builtin_memcpy(&t, &u, sizeof t);
    return t;
}

#define INFINITY __builtin_inff()

// threadgroup barriers of the threadgroup running now (oracle/metal_emu.cpp)
extern "C" void metal_shim_barrier(void);

namespace metal {
enum class mem_flags { mem_none, mem_device, mem_threadgroup };
inline void threadgroup_barrier(mem_flags) { metal_shim_barrier(); }
inline float exp(float x) { return __builtin_expf(x); }
inline float log(float x) { return __builtin_logf(x); }
inline float sqrt(float x) { return __builtin_sqrtf(x); }
inline float rsqrt(float x) { return 1.0f / __builtin_sqrtf(x); }
inline float pow(float a, float b) { return __builtin_powf(a, b); }
inline float sin(float x) { return __builtin_sinf(x); }
inline float cos(float x) { return __builtin_cosf(x); }
inline float fabs(float x) { return __builtin_fabsf(x); }
template <class T>
inline T min(T a, T b) { return b < a ? b : a; }
template <class T>
inline T max(T a, T b) { return a < b ? b : a; }
}  // namespace metal
