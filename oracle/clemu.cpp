// clemu.cpp -- TEST INFRASTRUCTURE ONLY: fiber-based work-groups for clemu.h.
//
// Each work-item runs on its own small stack.  barrier() saves the callee-saved registers and
// the stack pointer of the current fiber and switches back to the scheduler, which resumes the
// next unfinished fiber; one scheduler pass = one barrier interval for the whole work-group.
#include "clemu.h"

#include <cstdio>
#include <vector>

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
    tls_wg = saved;
}

}  // namespace clemu
