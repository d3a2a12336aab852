// msl_runtime.cpp -- execution model behind msl_shim.hpp: threadgroups of
// cooperative fibers on one OS thread, threadgroup barriers and SIMD-group
// collectives as rendezvous points, and the threadgroup-memory arenas.
// TEST INFRASTRUCTURE ONLY.
#include "msl_runtime.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

// Context switch (System V x86-64): save the callee-saved registers and the
// stack pointer of the running context, load the other one.
extern "C" void msl_ctx_switch(void** save_sp, void* load_sp);
extern "C" void msl_fiber_trampoline();
asm(R"(
    .text
    .globl msl_ctx_switch
    .type msl_ctx_switch,@function
msl_ctx_switch:
    pushq %rbp
    pushq %rbx
    pushq %r12
    pushq %r13
    pushq %r14
    pushq %r15
    movq %rsp, (%rdi)
    movq %rsi, %rsp
    popq %r15
    popq %r14
    popq %r13
    popq %r12
    popq %rbx
    popq %rbp
    ret
    .size msl_ctx_switch,.-msl_ctx_switch
    .globl msl_fiber_trampoline
    .type msl_fiber_trampoline,@function
msl_fiber_trampoline:
    movq %r12, %rdi
    callq *%r13
    ud2
    .size msl_fiber_trampoline,.-msl_fiber_trampoline
)");

namespace msl {

// exp(x): the oracle's method (Cody & Waite reduction with k read from
// fma(x, log2e, 1.5*2^23), degree-6 minimax polynomial, exact two-step
// scale), so every side evaluates the same bits.
float ref_expf(float x)
{
    if (x != x) return x + x;
    if (x > 88.72283935546875f) return __builtin_inff();
    if (x < -103.97208404541015625f) return 0.0f;
    const float log2e = 1.44269502162933349609375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187045e-06f;
    const float round_const = 12582912.0f;
    const float t = fmaf(x, log2e, round_const);
    const float k = t - round_const;
    float r = fmaf(-k, ln2_hi, x);
    r = fmaf(-k, ln2_lo, r);
    float p = 0.0013814594130963087f;
    p = fmaf(p, r, 0.0083687193691730499f);
    p = fmaf(p, r, 0.041668388992547989f);
    p = fmaf(p, r, 0.1666652113199234f);
    p = fmaf(p, r, 0.49999994039535522f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    uint32_t tb;
    std::memcpy(&tb, &t, 4);
    const int ki = (int)(tb - 0x4B400000u);
    const int e1 = ki / 2, e2 = ki - e1;
    auto pow2 = [](int e) {
        uint32_t u = (uint32_t)(e + 127) << 23;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    };
    return (p * pow2(e1)) * pow2(e2);
}

// ------------------------------------------------------------ launches
static std::atomic<unsigned long long> g_launch_gen{1};
unsigned long long tg_launch_generation() { return g_launch_gen.load(std::memory_order_relaxed); }
void begin_launch() { g_launch_gen.fetch_add(1); }

struct TgArray {
    void* p;
    std::size_t bytes;
};
static thread_local std::vector<TgArray> t_arrays;
static thread_local unsigned long long t_arrays_gen = 0;

void tg_register(void* p, std::size_t bytes)
{
    const unsigned long long g = tg_launch_generation();
    if (t_arrays_gen != g) {
        t_arrays.clear();
        t_arrays_gen = g;
    }
    t_arrays.push_back({p, bytes});
}

static void fill_tg_arrays()
{
    if (t_arrays_gen != tg_launch_generation()) return;
    for (auto& a : t_arrays) std::memset(a.p, 0x7F, a.bytes);
}

// -------------------------------------------------------------- fibers
constexpr std::size_t kStack = 64 * 1024;

struct Fiber {
    void* sp = nullptr;
    char* stack = nullptr;
    bool done = false;
    ThreadIds ids;
};

struct SimdGroup {
    int nlive = 0;
    int arrived = 0;
    unsigned gen = 0;
    uint32_t present[2] = {0, 0};
    uint32_t word[2][32];
};

struct Sched {
    void* main_sp = nullptr;
    std::vector<Fiber> fibers;
    int n = 0;
    int cur = -1;
    int nlive = 0;
    int bar_arrived = 0;
    unsigned bar_gen = 0;
    unsigned long long progress = 0;
    SimdGroup sg[32];
    const ThreadFn* fn = nullptr;
};
static thread_local Sched t_s;

static void yield_to_scheduler()
{
    Fiber& f = t_s.fibers[t_s.cur];
    msl_ctx_switch(&f.sp, t_s.main_sp);
}

static void release_simd(SimdGroup& s)
{
    s.arrived = 0;
    s.gen++;
    s.present[s.gen & 1] = 0;  // buffer of the next collective
}

extern "C" void msl_fiber_main(Fiber* f)
{
    (*t_s.fn)(f->ids);
    f->done = true;
    t_s.progress++;
    t_s.nlive--;
    if (t_s.bar_arrived > 0 && t_s.bar_arrived == t_s.nlive) {
        t_s.bar_arrived = 0;
        t_s.bar_gen++;
    }
    SimdGroup& s = t_s.sg[f->ids.sgid];
    s.nlive--;
    if (s.arrived > 0 && s.arrived == s.nlive) release_simd(s);
    msl_ctx_switch(&f->sp, t_s.main_sp);
    std::abort();  // never resumed
}

static void init_fiber(Fiber& f)
{
    if (!f.stack) f.stack = (char*)std::malloc(kStack);
    uintptr_t top = ((uintptr_t)(f.stack + kStack)) & ~(uintptr_t)15;
    void** sp = (void**)(top - 72);
    sp[0] = nullptr;                               // r15
    sp[1] = nullptr;                               // r14
    sp[2] = (void*)&msl_fiber_main;                // r13: entry
    sp[3] = (void*)&f;                             // r12: argument
    sp[4] = nullptr;                               // rbx
    sp[5] = nullptr;                               // rbp
    sp[6] = (void*)&msl_fiber_trampoline;          // return address
    f.sp = (void*)sp;
    f.done = false;
}

void run_threadgroup(const ThreadIds* ids, int n, const ThreadFn& fn)
{
    Sched& S = t_s;
    if ((int)S.fibers.size() < n) S.fibers.resize(n);
    S.n = n;
    S.fn = &fn;
    S.nlive = n;
    S.bar_arrived = 0;
    for (int k = 0; k < 32; k++) {
        S.sg[k].nlive = 0;
        S.sg[k].arrived = 0;
        S.sg[k].present[0] = S.sg[k].present[1] = 0;
    }
    for (int i = 0; i < n; i++) {
        S.fibers[i].ids = ids[i];
        init_fiber(S.fibers[i]);
        S.sg[ids[i].sgid].nlive++;
    }
    fill_tg_arrays();
    int remaining = n;
    while (remaining > 0) {
        const unsigned long long before = S.progress;
        remaining = 0;
        for (int i = 0; i < n; i++) {
            Fiber& f = S.fibers[i];
            if (f.done) continue;
            S.cur = i;
            msl_ctx_switch(&S.main_sp, f.sp);
            if (!f.done) remaining++;
        }
        if (remaining > 0 && S.progress == before) {
            std::fprintf(stderr, "msl shim: threadgroup deadlock (%d threads waiting)\n", remaining);
            std::abort();
        }
    }
    S.cur = -1;
}

// -------------------------------------------------------- collectives
void threadgroup_barrier(mem_flags)
{
    Sched& S = t_s;
    if (S.cur < 0) return;
    S.progress++;
    const unsigned g = S.bar_gen;
    if (++S.bar_arrived == S.nlive) {
        S.bar_arrived = 0;
        S.bar_gen++;
        return;
    }
    while (S.bar_gen == g) yield_to_scheduler();
}

// Rendezvous of the live lanes of the caller's SIMD group; returns the
// buffer index holding every present lane's word.
static int simd_exchange(uint32_t word, int& lane_out, uint32_t& present_out)
{
    Sched& S = t_s;
    Fiber& f = S.fibers[S.cur];
    SimdGroup& s = S.sg[f.ids.sgid];
    const int lane = (int)f.ids.lane;
    const unsigned g = s.gen;
    const int b = g & 1;
    s.word[b][lane] = word;
    s.present[b] |= 1u << lane;
    S.progress++;
    if (++s.arrived == s.nlive) {
        release_simd(s);
    } else {
        while (s.gen == g) yield_to_scheduler();
    }
    lane_out = lane;
    present_out = s.present[b];
    return b;
}

static SimdGroup& my_sg() { return t_s.sg[t_s.fibers[t_s.cur].ids.sgid]; }

template <class T>
static uint32_t to_word(T v)
{
    uint32_t w;
    std::memcpy(&w, &v, 4);
    return w;
}
template <class T>
static T from_word(uint32_t w)
{
    T v;
    std::memcpy(&v, &w, 4);
    return v;
}

float simd_sum(float v)
{
    int lane;
    uint32_t pres;
    const int b = simd_exchange(to_word(v), lane, pres);
    SimdGroup& s = my_sg();
    float acc = 0.f;
    bool first = true;
    for (int l = 0; l < 32; l++)
        if (pres >> l & 1) {
            const float x = from_word<float>(s.word[b][l]);
            acc = first ? x : acc + x;
            first = false;
        }
    return acc;
}

int simd_sum(int v)
{
    int lane;
    uint32_t pres;
    const int b = simd_exchange(to_word(v), lane, pres);
    SimdGroup& s = my_sg();
    int acc = 0;
    for (int l = 0; l < 32; l++)
        if (pres >> l & 1) acc += from_word<int>(s.word[b][l]);
    return acc;
}

int simd_max(int v)
{
    int lane;
    uint32_t pres;
    const int b = simd_exchange(to_word(v), lane, pres);
    SimdGroup& s = my_sg();
    int acc = v;
    for (int l = 0; l < 32; l++)
        if (pres >> l & 1) acc = std::max(acc, from_word<int>(s.word[b][l]));
    return acc;
}

int simd_or(int v)
{
    int lane;
    uint32_t pres;
    const int b = simd_exchange(to_word(v), lane, pres);
    SimdGroup& s = my_sg();
    int acc = 0;
    for (int l = 0; l < 32; l++)
        if (pres >> l & 1) acc |= from_word<int>(s.word[b][l]);
    return acc;
}

int simd_prefix_exclusive_sum(int v)
{
    int lane;
    uint32_t pres;
    const int b = simd_exchange(to_word(v), lane, pres);
    SimdGroup& s = my_sg();
    int acc = 0;
    for (int l = 0; l < lane; l++)
        if (pres >> l & 1) acc += from_word<int>(s.word[b][l]);
    return acc;
}

static uint32_t broadcast_word(uint32_t w, uint src)
{
    int lane;
    uint32_t pres;
    const int b = simd_exchange(w, lane, pres);
    SimdGroup& s = my_sg();
    if (src < 32 && (pres >> src & 1)) return s.word[b][src];
    for (int l = 0; l < 32; l++)
        if (pres >> l & 1) return s.word[b][l];
    return w;
}

float simd_broadcast(float v, uint lane) { return from_word<float>(broadcast_word(to_word(v), lane)); }
int simd_broadcast(int v, uint lane) { return from_word<int>(broadcast_word(to_word(v), lane)); }

}  // namespace msl
