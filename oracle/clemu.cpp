// clemu.cpp -- TEST INFRASTRUCTURE ONLY: fiber-based work-groups for clemu.h.
//
// Each work-item runs on its own small stack.  barrier() saves the callee-saved registers and
// the stack pointer of the current fiber and switches back to the scheduler, which resumes the
// next unfinished fiber; one scheduler pass = one barrier interval for the whole work-group.
#include "clemu.h"

#include <cstdio>
#include <vector>

#include <omp.h>
#include <sys/mman.h>

#if !defined(__x86_64__)
#include <ucontext.h>
#endif

namespace clemu {

thread_local WorkGroup* tls_wg = nullptr;

namespace {
constexpr size_t kStackBytes = 128 * 1024;

#if defined(__x86_64__)
// switch_stack(save, load): push callee-saved registers, store rsp into *save, load rsp from
// `load`, pop the registers saved there and return into that context.
extern "C" void clemu_switch(void** save, void* load);
asm(R"(
.text
.globl clemu_switch
.type clemu_switch,@function
clemu_switch:
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
.size clemu_switch,.-clemu_switch
)");

extern "C" void clemu_fiber_entry() {
    WorkGroup* wg = tls_wg;
    wg->body();
    wg->fibers[wg->cur].done = true;
    void* dummy;
    clemu_switch(&dummy, wg->sched_sp);
    std::abort();  // never resumed
}

void* init_stack(char* stack) {
    uintptr_t top = ((uintptr_t)(stack + kStackBytes)) & ~(uintptr_t)15;
    void** sp = (void**)top;
    *--sp = nullptr;                           // fake return address of the entry frame
    *--sp = (void*)&clemu_fiber_entry;         // popped by `ret`
    for (int i = 0; i < 6; ++i) *--sp = nullptr;  // rbp rbx r12 r13 r14 r15
    return (void*)sp;
}

inline void to_fiber(WorkGroup* wg, int i) { clemu_switch(&wg->sched_sp, wg->fibers[i].sp); }
inline void to_sched(WorkGroup* wg) { clemu_switch(&wg->fibers[wg->cur].sp, wg->sched_sp); }
#else
thread_local ucontext_t tls_sched_ctx;
thread_local std::vector<ucontext_t> tls_ctx;
void fiber_entry_uc() {
    WorkGroup* wg = tls_wg;
    wg->body();
    wg->fibers[wg->cur].done = true;
    swapcontext(&tls_ctx[wg->cur], &tls_sched_ctx);
}
#endif

struct FiberPool {
    std::vector<char*> stacks;
    std::vector<Fiber> fibers;
    ~FiberPool() { for (char* s : stacks) std::free(s); }
    void ensure(int n) {
        while ((int)stacks.size() < n) stacks.push_back((char*)std::malloc(kStackBytes));
        fibers.resize(n);
    }
};
thread_local FiberPool tls_pool;
}  // namespace

void barrier(int) {
    WorkGroup* wg = tls_wg;
#if defined(__x86_64__)
    to_sched(wg);
#else
    swapcontext(&tls_ctx[wg->cur], &tls_sched_ctx);
#endif
}

void run_work_group(size_t gx, size_t gy, size_t lx, size_t ly, const std::function<void()>& body) {
    const int n = (int)(lx * ly);
    tls_pool.ensure(n);
    WorkGroup wg;
    wg.n = n;
    wg.group_id[0] = gx;
    wg.group_id[1] = gy;
    wg.local_size[0] = lx;
    wg.local_size[1] = ly;
    wg.fibers = tls_pool.fibers.data();
    wg.body = body;
    WorkGroup* saved = tls_wg;
    tls_wg = &wg;
#if defined(__x86_64__)
    for (int i = 0; i < n; ++i) {
        wg.fibers[i].done = false;
        wg.fibers[i].stack = tls_pool.stacks[i];
        wg.fibers[i].sp = init_stack(tls_pool.stacks[i]);
    }
#else
    tls_ctx.resize(n);
    for (int i = 0; i < n; ++i) {
        wg.fibers[i].done = false;
        getcontext(&tls_ctx[i]);
        tls_ctx[i].uc_stack.ss_sp = tls_pool.stacks[i];
        tls_ctx[i].uc_stack.ss_size = kStackBytes;
        tls_ctx[i].uc_link = nullptr;
        makecontext(&tls_ctx[i], fiber_entry_uc, 0);
    }
#endif
    int remaining = n;
    while (remaining > 0) {
        for (int i = 0; i < n; ++i) {
            if (wg.fibers[i].done) continue;
            wg.cur = i;
#if defined(__x86_64__)
            to_fiber(&wg, i);
#else
            swapcontext(&tls_sched_ctx, &tls_ctx[i]);
#endif
            if (wg.fibers[i].done) --remaining;
        }
    }
    wg.free_locals();
    tls_wg = saved;
}

void run_work_groups_lockstep(size_t n_groups, size_t lx, const std::function<void()>& body, int n_threads) {
#if defined(__x86_64__)
    const int nt = n_threads > 0 ? n_threads : 1;
    std::vector<long> live((size_t)nt, 0);
    #pragma omp parallel num_threads(nt)
    {
        const size_t t = (size_t)omp_get_thread_num(), T = (size_t)omp_get_num_threads();
        std::vector<WorkGroup> wgs;
        for (size_t g = t; g < n_groups; g += T) {
            WorkGroup wg;
            wg.n = (int)lx;
            wg.group_id[0] = g;
            wg.local_size[0] = lx;
            wg.body = body;
            wgs.push_back(wg);
        }
        const size_t n_fibers = wgs.size() * lx;
        // one reservation for all stacks of this thread: pages are committed only when touched
        char* stacks = n_fibers ? (char*)mmap(nullptr, n_fibers * kStackBytes, PROT_READ | PROT_WRITE,
                                               MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0) : nullptr;
        if (n_fibers && stacks == (char*)MAP_FAILED) std::abort();
        std::vector<Fiber> fibers(n_fibers);
        for (size_t k = 0; k < wgs.size(); ++k) {
            wgs[k].fibers = fibers.data() + k * lx;
            for (size_t i = 0; i < lx; ++i) {
                Fiber& f = wgs[k].fibers[i];
                f.stack = stacks + (k * lx + i) * kStackBytes;
                f.sp = init_stack(f.stack);
                f.done = false;
            }
        }
        long mine = (long)n_fibers;
        for (;;) {
            for (WorkGroup& wg : wgs) {        // one barrier interval of every group of this thread
                tls_wg = &wg;
                for (int i = 0; i < wg.n; ++i) {
                    if (wg.fibers[i].done) continue;
                    wg.cur = i;
                    to_fiber(&wg, i);
                    if (wg.fibers[i].done) --mine;
                }
            }
            tls_wg = nullptr;
            live[t] = mine;
            #pragma omp barrier
            long total = 0;
            for (long x : live) total += x;
            #pragma omp barrier
            if (total == 0) break;
        }
        for (WorkGroup& wg : wgs) wg.free_locals();
        if (stacks) munmap(stacks, n_fibers * kStackBytes);
    }
#else
    (void)n_groups; (void)lx; (void)body; (void)n_threads;
    std::abort();   // lockstep scheduling is implemented for x86-64 only
#endif
}

}  // namespace clemu
