// msl_shim.hpp -- just enough of the Metal Shading Language, in C++20, to
// compile msplat's own kernels (core/metal/msplat_metal.metal) on the CPU.
// TEST INFRASTRUCTURE ONLY (the reference build that pins the oracle).
//
// Semantics chosen where the language leaves them to the GPU:
//   * arithmetic is IEEE float with no contraction (-ffp-contract=off); fma()
//     is fmaf; exp() is the shared Cody-Waite/Taylor msp_expf (the same
//     method the oracle and the CUDA engine use); sqrt/division are IEEE;
//     rsqrt(x) is 1/sqrt(x); vector ops are component-wise; matrix products
//     sum k = 0, 1, 2 left to right;
//   * threads of a threadgroup run as cooperative fibers on one OS thread;
//     threadgroup_barrier and the simd_* collectives are rendezvous points
//     over the threads that have not returned (Metal's active threads);
//   * threadgroup arrays are filled with 0x7F bytes before every
//     threadgroup, so a read of memory no thread wrote sees a large value
//     instead of the previous threadgroup's data;
//   * simd_broadcast from a lane that has returned yields the value of the
//     lowest lane still running.
#pragma once
#include <atomic>
#include <cstdint>
#include <cstring>
#include <type_traits>

extern "C" float sqrtf(float);
extern "C" float ceilf(float);
extern "C" float fmaf(float, float, float);
extern "C" float fabsf(float);
extern "C" float fminf(float, float);
extern "C" float fmaxf(float, float);
extern "C" float rintf(float);

namespace msl {

// ---------------------------------------------------------------- scalars
typedef unsigned int uint;
using std::int32_t;
using std::int64_t;
using std::uint32_t;
using std::uint64_t;

float ref_expf(float x);  // defined in msl_runtime.cpp (same method as the oracle)

inline float exp(float x) { return ref_expf(x); }
inline float sqrt(float x) { return sqrtf(x); }
inline float rsqrt(float x) { return 1.0f / sqrtf(x); }
inline float ceil(float x) { return ceilf(x); }
inline float fabs(float x) { return fabsf(x); }
inline float fma(float a, float b, float c) { return fmaf(a, b, c); }
inline float min(float a, float b) { return fminf(a, b); }
inline float max(float a, float b) { return fmaxf(a, b); }
inline int min(int a, int b) { return a < b ? a : b; }
inline int max(int a, int b) { return a > b ? a : b; }
inline uint min(uint a, uint b) { return a < b ? a : b; }
inline uint max(uint a, uint b) { return a > b ? a : b; }
inline float saturate(float x) { return fminf(fmaxf(x, 0.f), 1.f); }

template <class To, class From>
inline To as_type(From f)
{
    static_assert(sizeof(To) == sizeof(From), "as_type size");
    To t;
    std::memcpy(&t, &f, sizeof(To));
    return t;
}

// ---------------------------------------------------------------- vectors
template <class T, int N>
struct vec;

template <class T>
struct vec<T, 2> {
    T x, y;
    constexpr vec() : x(), y() {}
    constexpr vec(T a, T b) : x(a), y(b) {}
    template <class U>
    explicit constexpr vec(const vec<U, 2>& o) : x((T)o.x), y((T)o.y) {}
    T& operator[](int i) { return i == 0 ? x : y; }
    const T& operator[](int i) const { return i == 0 ? x : y; }
};
template <class T>
struct vec<T, 3> {
    T x, y, z;
    constexpr vec() : x(), y(), z() {}
    constexpr vec(T a, T b, T c) : x(a), y(b), z(c) {}
    explicit constexpr vec(T s) : x(s), y(s), z(s) {}
    template <class U>
    explicit constexpr vec(const vec<U, 3>& o) : x((T)o.x), y((T)o.y), z((T)o.z) {}
    T& operator[](int i) { return i == 0 ? x : (i == 1 ? y : z); }
    const T& operator[](int i) const { return i == 0 ? x : (i == 1 ? y : z); }
};
template <class T>
struct vec<T, 4> {
    T x, y, z, w;
    constexpr vec() : x(), y(), z(), w() {}
    constexpr vec(T a, T b, T c, T d) : x(a), y(b), z(c), w(d) {}
    template <class U>
    explicit constexpr vec(const vec<U, 4>& o) : x((T)o.x), y((T)o.y), z((T)o.z), w((T)o.w) {}
    T& operator[](int i) { return i == 0 ? x : (i == 1 ? y : (i == 2 ? z : w)); }
    const T& operator[](int i) const { return i == 0 ? x : (i == 1 ? y : (i == 2 ? z : w)); }
};

typedef vec<float, 2> float2;
typedef vec<float, 3> float3;
typedef vec<float, 4> float4;
typedef vec<int, 2> int2;
typedef vec<int, 3> int3;
typedef vec<uint, 2> uint2;
typedef vec<uint, 3> uint3;
typedef vec<uint, 4> uint4;

#define MSL_VEC_BINOP(OP)                                                           \
    template <class T, int N>                                                       \
    inline vec<T, N> operator OP(const vec<T, N>& a, const vec<T, N>& b)            \
    {                                                                               \
        vec<T, N> r;                                                                \
        for (int i = 0; i < N; i++) r[i] = a[i] OP b[i];                            \
        return r;                                                                   \
    }                                                                               \
    template <class T, int N, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> \
    inline vec<T, N> operator OP(const vec<T, N>& a, S s)                           \
    {                                                                               \
        vec<T, N> r;                                                                \
        for (int i = 0; i < N; i++) r[i] = a[i] OP (T)s;                            \
        return r;                                                                   \
    }                                                                               \
    template <class T, int N, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> \
    inline vec<T, N> operator OP(S s, const vec<T, N>& a)                           \
    {                                                                               \
        vec<T, N> r;                                                                \
        for (int i = 0; i < N; i++) r[i] = (T)s OP a[i];                            \
        return r;                                                                   \
    }                                                                               \
    template <class T, int N>                                                       \
    inline vec<T, N>& operator OP##=(vec<T, N>& a, const vec<T, N>& b)              \
    {                                                                               \
        for (int i = 0; i < N; i++) a[i] = a[i] OP b[i];                            \
        return a;                                                                   \
    }                                                                               \
    template <class T, int N, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> \
    inline vec<T, N>& operator OP##=(vec<T, N>& a, S s)                             \
    {                                                                               \
        for (int i = 0; i < N; i++) a[i] = a[i] OP (T)s;                            \
        return a;                                                                   \
    }
MSL_VEC_BINOP(+)
MSL_VEC_BINOP(-)
MSL_VEC_BINOP(*)
MSL_VEC_BINOP(/)
#undef MSL_VEC_BINOP

template <class T, int N>
inline vec<T, N> operator-(const vec<T, N>& a)
{
    vec<T, N> r;
    for (int i = 0; i < N; i++) r[i] = -a[i];
    return r;
}

template <int N>
inline vec<float, N> max(const vec<float, N>& a, float s)
{
    vec<float, N> r;
    for (int i = 0; i < N; i++) r[i] = fmaxf(a[i], s);
    return r;
}
template <int N>
inline vec<float, N> min(const vec<float, N>& a, float s)
{
    vec<float, N> r;
    for (int i = 0; i < N; i++) r[i] = fminf(a[i], s);
    return r;
}
template <int N>
inline vec<float, N> exp(const vec<float, N>& a)
{
    vec<float, N> r;
    for (int i = 0; i < N; i++) r[i] = ref_expf(a[i]);
    return r;
}
template <int N>
inline vec<float, N> saturate(const vec<float, N>& a)
{
    vec<float, N> r;
    for (int i = 0; i < N; i++) r[i] = saturate(a[i]);
    return r;
}
template <int N>
inline vec<float, N> fma(const vec<float, N>& a, const vec<float, N>& b, const vec<float, N>& c)
{
    vec<float, N> r;
    for (int i = 0; i < N; i++) r[i] = fmaf(a[i], b[i], c[i]);
    return r;
}
template <int N>
inline vec<float, N> fma(const vec<float, N>& a, float b, const vec<float, N>& c)
{
    vec<float, N> r;
    for (int i = 0; i < N; i++) r[i] = fmaf(a[i], b, c[i]);
    return r;
}
inline float dot(const float2& a, const float2& b) { return a.x * b.x + a.y * b.y; }
inline float dot(const float3& a, const float3& b) { return (a.x * b.x + a.y * b.y) + a.z * b.z; }
inline float3 normalize(const float3& v) { return v * rsqrt(dot(v, v)); }

// --------------------------------------------------------------- matrices
template <int N>
struct matf {
    vec<float, N> c[N];  // columns
    matf() {}
    explicit matf(float d)
    {
        for (int i = 0; i < N; i++)
            for (int j = 0; j < N; j++) c[i][j] = i == j ? d : 0.f;
    }
    template <class... A, class = std::enable_if_t<sizeof...(A) == N * N>>
    matf(A... a)
    {
        const float v[N * N] = {(float)a...};
        for (int i = 0; i < N; i++)
            for (int j = 0; j < N; j++) c[i][j] = v[i * N + j];
    }
    vec<float, N>& operator[](int i) { return c[i]; }
    const vec<float, N>& operator[](int i) const { return c[i]; }
};
typedef matf<2> float2x2;
typedef matf<3> float3x3;

template <int N>
inline matf<N> operator*(const matf<N>& A, const matf<N>& B)
{
    matf<N> C(0.f);
    for (int col = 0; col < N; col++)
        for (int r = 0; r < N; r++) {
            float s = A[0][r] * B[col][0];
            for (int k = 1; k < N; k++) s = s + A[k][r] * B[col][k];
            C[col][r] = s;
        }
    return C;
}
template <int N, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>>
inline matf<N> operator*(S s, const matf<N>& A)
{
    matf<N> C(0.f);
    for (int i = 0; i < N; i++)
        for (int j = 0; j < N; j++) C[i][j] = (float)s * A[i][j];
    return C;
}
template <int N>
inline matf<N> operator+(const matf<N>& A, const matf<N>& B)
{
    matf<N> C(0.f);
    for (int i = 0; i < N; i++)
        for (int j = 0; j < N; j++) C[i][j] = A[i][j] + B[i][j];
    return C;
}
template <int N>
inline matf<N> transpose(const matf<N>& A)
{
    matf<N> T(0.f);
    for (int i = 0; i < N; i++)
        for (int j = 0; j < N; j++) T[i][j] = A[j][i];
    return T;
}

// ----------------------------------------------------------------- atomics
typedef std::atomic<float> atomic_float;
typedef std::atomic<uint> atomic_uint;
using memory_order = std::memory_order;
using std::memory_order_relaxed;
inline float atomic_fetch_add_explicit(atomic_float* p, float v, memory_order o) { return p->fetch_add(v, o); }
inline uint atomic_fetch_add_explicit(atomic_uint* p, uint v, memory_order o) { return p->fetch_add(v, o); }
inline void atomic_store_explicit(atomic_uint* p, uint v, memory_order o) { p->store(v, o); }
inline uint atomic_load_explicit(atomic_uint* p, memory_order o) { return p->load(o); }

// -------------------------------------------------- threadgroup execution
enum class mem_flags { mem_none, mem_threadgroup, mem_device, mem_texture };

void threadgroup_barrier(mem_flags);
void tg_register(void* p, std::size_t bytes);
unsigned long long tg_launch_generation();

// Storage of one `threadgroup` declaration.  Shared by the fibers of a
// threadgroup (they run on one OS thread); filled with 0x7F bytes when first
// used in a launch and before every later threadgroup of that launch.
template <class T, int ID>
inline T& tg_array()
{
    static thread_local T storage;
    static thread_local unsigned long long gen = 0;
    const unsigned long long g = tg_launch_generation();
    if (gen != g) {
        gen = g;
        std::memset((void*)&storage, 0x7F, sizeof(T));
        tg_register((void*)&storage, sizeof(T));
    }
    return storage;
}

// SIMD-group collectives over the lanes that have not returned.
float simd_sum(float v);
int simd_sum(int v);
int simd_max(int v);
int simd_or(int v);
int simd_prefix_exclusive_sum(int v);
float simd_broadcast(float v, uint lane);
int simd_broadcast(int v, uint lane);
inline float3 simd_broadcast(float3 v, uint lane)
{
    return float3(simd_broadcast(v.x, lane), simd_broadcast(v.y, lane), simd_broadcast(v.z, lane));
}

}  // namespace msl
