// cl_cpu.cpp -- an OpenCL 1.1 host runtime on the CPU, just large enough to
// run the reference's main.c with its own kernels.
//
// TEST INFRASTRUCTURE ONLY.  The reference (GPT2-OpenCL-1.1) needs an
// OpenCL platform, and none exists here or on the GPU box.  This file gives
// main.c one "GPU" device whose kernels are the reference's math.cl (and the
// matmul source main.c generates at main.c:593-684) compiled ahead of time as
// C++ with mathcl_prelude.h.  Buffers are host memory; the queue executes
// each command when it is enqueued (the reference only uses an in-order
// queue with blocking transfers).
//
// Work-items: kernels without barriers run one work-item per call with the
// work-item ids in thread-local storage, spread over OpenMP threads.
// Kernels with barriers (attn_softmax_1q, matmul) run their work-groups in
// parallel over OpenMP threads; within a group each work-item is a fiber on
// its own small stack, and barrier() switches back to the group's scheduler,
// which resumes every fiber in turn (a barrier is reached by all work-items
// before any passes it).  __local arrays are thread_local statics, so each
// thread's group has its own.  The switch saves only the callee-saved
// registers and the stack pointer (x86-64 System V).
#include "CL/cl.h"

#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

struct float4;   // only passed through as a pointer

// ---- kernels compiled from the reference's sources (extern "C") -----------
extern "C" {
void matmul(const float *, const float *, const float *, float *, int, int, int, int);
void matvec(const float *, const float *, const float *, const float *, float *, int, int, int);
void matvec4(const float *, const float4 *, const float *, const float *, float *, int, int, int);
void matvec4_sk(const float *, const float4 *, float4 *, int, int, int);
void reduce_partial(const float4 *, const float *, const float *, float *, int, int, int);
void layernorm(const float *, float *, const float *, const float *, int, int);
void add_inplace(float *, const float *, int);
void gelu(float *, int);
void embed(const float *, const float *, float *, int, int, int, const int *);
void split_kv(const float *, float *, float *, int, int, int, int);
void attn_scores_1q(const float *, const float *, float *, int, int, int, int, int, int, float);
void attn_softmax_1q(float *, int);
void attn_out_1q(const float *, const float *, float *, int, int, int, int);
// main.c's runtime matmul for tile 64x64x16 / 4x4 (the one the reference's
// README run selected), renamed at compile time.
void refmm_64x64x16_4x4(const float *, const float *, const float *, float *, int, int, int, int);
}

// ---- work-item ids ------------------------------------------------------------
static thread_local size_t t_gid[3], t_lid[3], t_grp[3], t_lsz[3] = {1, 1, 1}, t_gsz[3] = {1, 1, 1};

// ---- fibers: one work-group's work-items on one OS thread -------------------------
extern "C" void g2ref_fiber_switch(void **save_sp, void *load_sp);
asm(R"(
    .text
    .globl g2ref_fiber_switch
    .type g2ref_fiber_switch,@function
g2ref_fiber_switch:
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
    .size g2ref_fiber_switch, .-g2ref_fiber_switch
)");

namespace {
typedef void (*thunk_fn)(const uint64_t *a);
constexpr size_t kFiberStack = 32 * 1024;
struct Fiber {
    void *sp;
    bool done;
    size_t lid[3];
};
thread_local std::vector<Fiber> t_fibers;
thread_local std::vector<char> t_stacks;
thread_local void *t_sched_sp = nullptr;
thread_local int t_cur = -1;             // running fiber, -1 outside a group
thread_local thunk_fn t_job = nullptr;
thread_local const uint64_t *t_job_args = nullptr;

[[noreturn]] void fiber_entry() {
    t_job(t_job_args);
    t_fibers[(size_t)t_cur].done = true;
    void *dead;
    g2ref_fiber_switch(&dead, t_sched_sp);   // never resumed
    __builtin_unreachable();
}
}  // namespace

extern "C" size_t get_global_id(unsigned d) { return d < 3 ? t_gid[d] : 0; }
extern "C" size_t get_local_id(unsigned d) { return d < 3 ? t_lid[d] : 0; }
extern "C" size_t get_group_id(unsigned d) { return d < 3 ? t_grp[d] : 0; }
extern "C" size_t get_local_size(unsigned d) { return d < 3 ? t_lsz[d] : 1; }
extern "C" size_t get_global_size(unsigned d) { return d < 3 ? t_gsz[d] : 1; }
extern "C" void barrier(int) {
    if (t_cur >= 0) g2ref_fiber_switch(&t_fibers[(size_t)t_cur].sp, t_sched_sp);
}
// Present in builds whose barrier kernels run on fibers (fast enough for the
// full-size model); the test harness checks for this symbol.
extern "C" int refcl_fiber_executor(void) { return 1; }

// ---- objects --------------------------------------------------------------------
struct _cl_platform_id { int dummy; };
struct _cl_device_id { int dummy; };
struct _cl_context { int refs; };
struct _cl_command_queue { int refs; };
struct _cl_mem {
    void *ptr;
    size_t size;
};
struct _cl_program {
    std::string src;
    std::string log;
    int kind;   // 0 = math.cl kernels, 1 = generated matmul 64x64x16/4x4, -1 = unbuildable
};
typedef void (*thunk_t)(const uint64_t *a);
struct _cl_kernel {
    std::string name;
    thunk_t fn;
    int barrier_kernel;
    int nargs;
    const char *kinds;   // per argument: 'm' buffer, 'i' int, 'f' float
    uint64_t raw[16];    // int/float bits, or the cl_mem handle
    bool set[16];
};

static _cl_platform_id g_platform;
static _cl_device_id g_device;

#define PF(i) ((float *)a[i])
#define CPF(i) ((const float *)a[i])
#define I(i) ((int)(int32_t)a[i])
static float F(uint64_t v) {
    uint32_t u = (uint32_t)v;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

struct KernelDef {
    const char *name;
    const char *kinds;
    thunk_t fn;
    int barrier_kernel;
    int program_kind;
};
static const KernelDef kDefs[] = {
    {"matmul", "mmmmiiii", [](const uint64_t *a) { matmul(CPF(0), CPF(1), CPF(2), PF(3), I(4), I(5), I(6), I(7)); }, 1, 0},
    {"matvec", "mmmmmiii", [](const uint64_t *a) { matvec(CPF(0), CPF(1), CPF(2), CPF(3), PF(4), I(5), I(6), I(7)); }, 0, 0},
    {"matvec4", "mmmmmiii", [](const uint64_t *a) { matvec4(CPF(0), (const float4 *)a[1], CPF(2), CPF(3), PF(4), I(5), I(6), I(7)); }, 0, 0},
    {"matvec4_sk", "mmmiii", [](const uint64_t *a) { matvec4_sk(CPF(0), (const float4 *)a[1], (float4 *)a[2], I(3), I(4), I(5)); }, 0, 0},
    {"reduce_partial", "mmmmiii", [](const uint64_t *a) { reduce_partial((const float4 *)a[0], CPF(1), CPF(2), PF(3), I(4), I(5), I(6)); }, 0, 0},
    {"layernorm", "mmmmii", [](const uint64_t *a) { layernorm(CPF(0), PF(1), CPF(2), CPF(3), I(4), I(5)); }, 0, 0},
    {"add_inplace", "mmi", [](const uint64_t *a) { add_inplace(PF(0), CPF(1), I(2)); }, 0, 0},
    {"gelu", "mi", [](const uint64_t *a) { gelu(PF(0), I(1)); }, 0, 0},
    {"embed", "mmmiiim", [](const uint64_t *a) { embed(CPF(0), CPF(1), PF(2), I(3), I(4), I(5), (const int *)a[6]); }, 0, 0},
    {"split_kv", "mmmiiii", [](const uint64_t *a) { split_kv(CPF(0), PF(1), PF(2), I(3), I(4), I(5), I(6)); }, 0, 0},
    {"attn_scores_1q", "mmmiiiiiif", [](const uint64_t *a) { attn_scores_1q(CPF(0), CPF(1), PF(2), I(3), I(4), I(5), I(6), I(7), I(8), F(a[9])); }, 0, 0},
    {"attn_softmax_1q", "mi", [](const uint64_t *a) { attn_softmax_1q(PF(0), I(1)); }, 1, 0},
    {"attn_out_1q", "mmmiiii", [](const uint64_t *a) { attn_out_1q(CPF(0), CPF(1), PF(2), I(3), I(4), I(5), I(6)); }, 0, 0},
    {"matmul", "mmmmiiii", [](const uint64_t *a) { refmm_64x64x16_4x4(CPF(0), CPF(1), CPF(2), PF(3), I(4), I(5), I(6), I(7)); }, 1, 1},
};

static void copy_str(const char *s, size_t size, void *value, size_t *size_ret) {
    size_t n = strlen(s) + 1;
    if (value && size) {
        size_t c = n < size ? n : size;
        memcpy(value, s, c);
        ((char *)value)[c - 1] = 0;
    }
    if (size_ret) *size_ret = n;
}
template <class T>
static void copy_val(T v, size_t size, void *value, size_t *size_ret) {
    if (value && size >= sizeof(T)) memcpy(value, &v, sizeof(T));
    if (size_ret) *size_ret = sizeof(T);
}

extern "C" {

cl_int clGetPlatformIDs(cl_uint n, cl_platform_id *p, cl_uint *np) {
    if (p && n) p[0] = &g_platform;
    if (np) *np = 1;
    return CL_SUCCESS;
}
cl_int clGetPlatformInfo(cl_platform_id, cl_platform_info name, size_t size, void *value, size_t *size_ret) {
    if (name != CL_PLATFORM_NAME) return CL_INVALID_VALUE;
    copy_str("gpt2b200 CPU shim", size, value, size_ret);
    return CL_SUCCESS;
}
cl_int clGetDeviceIDs(cl_platform_id, cl_device_type, cl_uint n, cl_device_id *d, cl_uint *nd) {
    if (d && n) d[0] = &g_device;
    if (nd) *nd = 1;
    return CL_SUCCESS;
}
cl_int clGetDeviceInfo(cl_device_id, cl_device_info name, size_t size, void *value, size_t *size_ret) {
    switch (name) {
    case CL_DEVICE_NAME: copy_str("host CPU (reference kernels)", size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_VENDOR: copy_str("gpt2b200 oracle", size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_EXTENSIONS: copy_str("cl_khr_fp64", size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_MAX_COMPUTE_UNITS: copy_val<cl_uint>((cl_uint)std::thread::hardware_concurrency(), size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_MAX_CLOCK_FREQUENCY: copy_val<cl_uint>(1000, size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_GLOBAL_MEM_SIZE: copy_val<cl_ulong>(64ull << 30, size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_LOCAL_MEM_SIZE: copy_val<cl_ulong>(48u << 10, size, value, size_ret); return CL_SUCCESS;
    case CL_DEVICE_MAX_WORK_GROUP_SIZE: copy_val<size_t>(1024, size, value, size_ret); return CL_SUCCESS;
    default: return CL_INVALID_VALUE;
    }
}
cl_context clCreateContext(const cl_context_properties *, cl_uint, const cl_device_id *,
                           void (*)(const char *, const void *, size_t, void *), void *, cl_int *err) {
    if (err) *err = CL_SUCCESS;
    return new _cl_context{1};
}
cl_command_queue clCreateCommandQueue(cl_context, cl_device_id, cl_command_queue_properties, cl_int *err) {
    if (err) *err = CL_SUCCESS;
    return new _cl_command_queue{1};
}
cl_program clCreateProgramWithSource(cl_context, cl_uint count, const char **strings, const size_t *lengths,
                                     cl_int *err) {
    auto *p = new _cl_program;
    for (cl_uint i = 0; i < count; ++i)
        p->src.append(strings[i], lengths && lengths[i] ? lengths[i] : strlen(strings[i]));
    p->kind = -1;
    if (err) *err = CL_SUCCESS;
    return p;
}
// A program is either the math.cl kernel set, or main.c's generated matmul,
// which exists here for the 64x64x16/4x4 tile only.
cl_int clBuildProgram(cl_program p, cl_uint, const cl_device_id *, const char *, void (*)(cl_program, void *), void *) {
    if (p->src.find("#define MM_BM") == std::string::npos) {
        p->kind = 0;
        return CL_SUCCESS;
    }
    int bm = 0, bn = 0, bk = 0, tm = 0, tn = 0;
    const char *s = p->src.c_str();
    const char *q;
    if ((q = strstr(s, "#define MM_BM "))) bm = atoi(q + 14);
    if ((q = strstr(s, "#define MM_BN "))) bn = atoi(q + 14);
    if ((q = strstr(s, "#define MM_BK "))) bk = atoi(q + 14);
    if ((q = strstr(s, "#define MM_TM "))) tm = atoi(q + 14);
    if ((q = strstr(s, "#define MM_TN "))) tn = atoi(q + 14);
    if (bm == 64 && bn == 64 && bk == 16 && tm == 4 && tn == 4) {
        p->kind = 1;
        return CL_SUCCESS;
    }
    p->log = "cpu shim: only the 64x64x16/4x4 matmul tile is compiled ahead of time";
    return CL_BUILD_PROGRAM_FAILURE;
}
cl_int clGetProgramBuildInfo(cl_program p, cl_device_id, cl_program_build_info name, size_t size, void *value,
                             size_t *size_ret) {
    if (name != CL_PROGRAM_BUILD_LOG) return CL_INVALID_VALUE;
    copy_str(p->log.c_str(), size, value, size_ret);
    return CL_SUCCESS;
}
cl_kernel clCreateKernel(cl_program p, const char *name, cl_int *err) {
    for (const auto &d : kDefs) {
        if (d.program_kind == p->kind && strcmp(d.name, name) == 0) {
            auto *k = new _cl_kernel;
            k->name = name;
            k->fn = d.fn;
            k->barrier_kernel = d.barrier_kernel;
            k->kinds = d.kinds;
            k->nargs = (int)strlen(d.kinds);
            memset(k->raw, 0, sizeof k->raw);
            memset(k->set, 0, sizeof k->set);
            if (err) *err = CL_SUCCESS;
            return k;
        }
    }
    if (err) *err = CL_INVALID_KERNEL_NAME;
    return nullptr;
}
cl_int clSetKernelArg(cl_kernel k, cl_uint idx, size_t size, const void *value) {
    if ((int)idx >= k->nargs) return CL_INVALID_ARG_INDEX;
    uint64_t v = 0;
    if (k->kinds[idx] == 'm') {
        if (size != sizeof(cl_mem)) return CL_INVALID_VALUE;
        cl_mem m = value ? *(const cl_mem *)value : nullptr;
        v = (uint64_t)(uintptr_t)m;
    } else {
        if (size != 4 || !value) return CL_INVALID_VALUE;
        uint32_t u;
        memcpy(&u, value, 4);
        v = u;
    }
    k->raw[idx] = v;
    k->set[idx] = true;
    return CL_SUCCESS;
}

// ---- work-groups with barriers: fibers on each OpenMP thread ---------------------
namespace {
// Run work-group (g0, g1, g2) of fn: every work-item a fiber, switched round robin.
void run_group(thunk_fn fn, const uint64_t *a, const size_t *l, const size_t *g, size_t g0, size_t g1, size_t g2) {
    const size_t n = l[0] * l[1] * l[2];
    if (t_fibers.size() < n) {
        t_fibers.resize(n);
        t_stacks.assign(n * kFiberStack + 64, 0);
    }
    char *base = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(t_stacks.data()) + 63) & ~(uintptr_t)63);
    for (size_t i = 0; i < n; ++i) {
        Fiber &f = t_fibers[i];
        // stack top 16-byte aligned; the first switch pops six zero registers and
        // returns into fiber_entry with rsp = 8 mod 16, as after a call
        uintptr_t top = (reinterpret_cast<uintptr_t>(base + (i + 1) * kFiberStack)) & ~(uintptr_t)15;
        uint64_t *sp = reinterpret_cast<uint64_t *>(top - 16);
        sp[0] = reinterpret_cast<uint64_t>(&fiber_entry);
        sp[1] = 0;
        sp -= 6;
        for (int r = 0; r < 6; ++r) sp[r] = 0;
        f.sp = sp;
        f.done = false;
        f.lid[0] = i % l[0];
        f.lid[1] = (i / l[0]) % l[1];
        f.lid[2] = i / (l[0] * l[1]);
    }
    t_job = fn;
    t_job_args = a;
    const size_t grp[3] = {g0, g1, g2};
    for (int d = 0; d < 3; ++d) {
        t_grp[d] = grp[d];
        t_lsz[d] = l[d];
        t_gsz[d] = g[d];
    }
    size_t left = n;
    while (left > 0) {
        for (size_t i = 0; i < n; ++i) {
            Fiber &f = t_fibers[i];
            if (f.done) continue;
            t_cur = (int)i;
            for (int d = 0; d < 3; ++d) {
                t_lid[d] = f.lid[d];
                t_gid[d] = grp[d] * l[d] + f.lid[d];
            }
            g2ref_fiber_switch(&t_sched_sp, f.sp);   // back at the fiber's next barrier or its end
            if (f.done) --left;
        }
    }
    t_cur = -1;
}
}  // namespace

cl_int clEnqueueNDRangeKernel(cl_command_queue, cl_kernel k, cl_uint dim, const size_t *off, const size_t *gws,
                              const size_t *lws, cl_uint, const cl_event *, cl_event *) {
    if (dim < 1 || dim > 3 || off) return CL_INVALID_VALUE;
    for (int i = 0; i < k->nargs; ++i)
        if (!k->set[i]) return CL_INVALID_KERNEL_ARGS;
    uint64_t a[16];
    for (int i = 0; i < k->nargs; ++i) {
        if (k->kinds[i] == 'm') {
            cl_mem m = (cl_mem)(uintptr_t)k->raw[i];
            a[i] = m ? (uint64_t)(uintptr_t)m->ptr : 0;
        } else {
            a[i] = k->raw[i];
        }
    }
    size_t g[3] = {1, 1, 1}, l[3] = {1, 1, 1};
    for (cl_uint d = 0; d < dim; ++d) {
        g[d] = gws[d];
        l[d] = lws ? lws[d] : 1;
        if (l[d] == 0 || g[d] % l[d]) return CL_INVALID_WORK_GROUP_SIZE;
    }
    if (k->barrier_kernel) {
        if (l[0] * l[1] * l[2] > 1024) return CL_INVALID_WORK_GROUP_SIZE;
        const long ng[3] = {(long)(g[0] / l[0]), (long)(g[1] / l[1]), (long)(g[2] / l[2])};
        const long groups = ng[0] * ng[1] * ng[2];
        thunk_fn fn = k->fn;
#pragma omp parallel for schedule(dynamic, 1)
        for (long q = 0; q < groups; ++q)
            run_group(fn, a, l, g, (size_t)(q % ng[0]), (size_t)((q / ng[0]) % ng[1]), (size_t)(q / (ng[0] * ng[1])));
        return CL_SUCCESS;
    }
    const long total = (long)(g[0] * g[1] * g[2]);
    thunk_t fn = k->fn;
#pragma omp parallel for schedule(static, 64)
    for (long w = 0; w < total; ++w) {
        size_t id[3] = {(size_t)w % g[0], ((size_t)w / g[0]) % g[1], (size_t)w / (g[0] * g[1])};
        for (int d = 0; d < 3; ++d) {
            t_gid[d] = id[d];
            t_lsz[d] = l[d];
            t_gsz[d] = g[d];
            t_lid[d] = id[d] % l[d];
            t_grp[d] = id[d] / l[d];
        }
        fn(a);
    }
    return CL_SUCCESS;
}
cl_int clFinish(cl_command_queue) { return CL_SUCCESS; }

cl_mem clCreateBuffer(cl_context, cl_mem_flags, size_t size, void *host_ptr, cl_int *err) {
    auto *m = new _cl_mem;
    m->size = size;
    m->ptr = calloc(size ? size : 1, 1);
    if (!m->ptr) {
        delete m;
        if (err) *err = CL_MEM_OBJECT_ALLOCATION_FAILURE;
        return nullptr;
    }
    if (host_ptr) memcpy(m->ptr, host_ptr, size);
    if (err) *err = CL_SUCCESS;
    return m;
}
cl_int clEnqueueWriteBuffer(cl_command_queue, cl_mem b, cl_bool, size_t off, size_t size, const void *ptr, cl_uint,
                            const cl_event *, cl_event *) {
    if (!b || off + size > b->size) return CL_INVALID_VALUE;
    memcpy((char *)b->ptr + off, ptr, size);
    return CL_SUCCESS;
}
cl_int clEnqueueReadBuffer(cl_command_queue, cl_mem b, cl_bool, size_t off, size_t size, void *ptr, cl_uint,
                           const cl_event *, cl_event *) {
    if (!b || off + size > b->size) return CL_INVALID_VALUE;
    memcpy(ptr, (const char *)b->ptr + off, size);
    return CL_SUCCESS;
}
cl_int clEnqueueWriteBufferRect(cl_command_queue, cl_mem b, cl_bool, const size_t *bo, const size_t *ho,
                                const size_t *region, size_t brp, size_t bsp, size_t hrp, size_t hsp,
                                const void *ptr, cl_uint, const cl_event *, cl_event *) {
    if (!brp) brp = region[0];
    if (!bsp) bsp = region[1] * brp;
    if (!hrp) hrp = region[0];
    if (!hsp) hsp = region[1] * hrp;
    for (size_t z = 0; z < region[2]; ++z)
        for (size_t y = 0; y < region[1]; ++y) {
            size_t boff = (bo[2] + z) * bsp + (bo[1] + y) * brp + bo[0];
            size_t hoff = (ho[2] + z) * hsp + (ho[1] + y) * hrp + ho[0];
            if (boff + region[0] > b->size) return CL_INVALID_VALUE;
            memcpy((char *)b->ptr + boff, (const char *)ptr + hoff, region[0]);
        }
    return CL_SUCCESS;
}
cl_int clEnqueueCopyBuffer(cl_command_queue, cl_mem s, cl_mem d, size_t so, size_t dof, size_t size, cl_uint,
                           const cl_event *, cl_event *) {
    if (!s || !d || so + size > s->size || dof + size > d->size) return CL_INVALID_VALUE;
    memmove((char *)d->ptr + dof, (const char *)s->ptr + so, size);
    return CL_SUCCESS;
}
cl_int clReleaseMemObject(cl_mem m) {
    if (!m) return CL_INVALID_MEM_OBJECT;
    free(m->ptr);
    delete m;
    return CL_SUCCESS;
}
cl_int clReleaseKernel(cl_kernel k) {
    delete k;
    return CL_SUCCESS;
}
cl_int clReleaseProgram(cl_program p) {
    delete p;
    return CL_SUCCESS;
}
cl_int clReleaseCommandQueue(cl_command_queue q) {
    delete q;
    return CL_SUCCESS;
}
cl_int clReleaseContext(cl_context c) {
    delete c;
    return CL_SUCCESS;
}

}   // extern "C"

// Direct access for per-kernel pin tests: run one named math.cl kernel over an
// NDRange with host pointers (kinds as in kDefs; scalars passed as 32-bit bits).
extern "C" int refcl_run_kernel(const char *name, int program_kind, int dim, const size_t *gws, const size_t *lws,
                                const uint64_t *args, int nargs) {
    cl_program p = new _cl_program;
    p->kind = program_kind;
    cl_int err;
    cl_kernel k = clCreateKernel(p, name, &err);
    delete p;
    if (!k) return err;
    if (nargs != k->nargs) { delete k; return CL_INVALID_KERNEL_ARGS; }
    std::vector<_cl_mem> mems((size_t)nargs);
    for (int i = 0; i < nargs; ++i) {
        if (k->kinds[i] == 'm') {
            if (args[i]) {
                mems[i].ptr = (void *)(uintptr_t)args[i];
                mems[i].size = (size_t)-1;
                cl_mem m = &mems[i];
                clSetKernelArg(k, (cl_uint)i, sizeof(cl_mem), &m);
            } else {
                clSetKernelArg(k, (cl_uint)i, sizeof(cl_mem), nullptr);
            }
        } else {
            uint32_t u = (uint32_t)args[i];
            clSetKernelArg(k, (cl_uint)i, 4, &u);
        }
    }
    err = clEnqueueNDRangeKernel(nullptr, k, (cl_uint)dim, nullptr, gws, lws, 0, nullptr, nullptr);
    delete k;
    return err;
}
