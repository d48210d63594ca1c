/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the work-group runner of cl_emul.h. Work-groups
 * run one after another on the calling thread (the kernels' local arrays
 * are statics, one per work-group). A group of one work-item runs as a
 * plain call; a group of L > 1 runs its work-items as L coroutines
 * (ucontext) on their own stacks, round robin: barrier() hands control to
 * the next work-item, so every work-item reaches a barrier before any
 * passes it, and each work-item's ids are swapped in with it. */

#include <stdlib.h>
#include <ucontext.h>

#include "cl_emul.h"

__thread struct emul_item emul_wi;

#define EMUL_STACK (256 * 1024)

static ucontext_t sched;
static ucontext_t *items_ctx;
static int in_group;
static int current;

void emul_barrier(void)
{
    if (in_group)
        swapcontext(&items_ctx[current], &sched);
}

struct emul_launch {
    void (*body)(void *);
    void *args;
    size_t g[3], l[3], ng[3];
};

static const struct emul_launch *launch;
static unsigned char *finished;

static void emul_set(struct emul_item *wi, const struct emul_launch *L, const size_t grp[3],
                     const size_t lid[3])
{
    for (int d = 0; d < 3; d++) {
        wi->grp[d] = grp[d];
        wi->lid[d] = lid[d];
        wi->gid[d] = grp[d] * L->l[d] + lid[d];
        wi->lsz[d] = L->l[d];
        wi->gsz[d] = L->g[d];
    }
}

/* A work-item: the kernel body, then back to the scheduler (uc_link). */
static void emul_item_main(void)
{
    launch->body(launch->args);
    finished[current] = 1;
}

void emul_launch(void (*body)(void *), void *args, const size_t g[3], const size_t l[3])
{
    struct emul_launch L;
    size_t items = 1, grp[3];

    L.body = body;
    L.args = args;
    for (int d = 0; d < 3; d++) {
        L.g[d] = g[d];
        L.l[d] = l[d];
        L.ng[d] = g[d] / l[d];
        items *= l[d];
    }
    if (items == 1) {
        const size_t lid[3] = {0, 0, 0};

        for (grp[2] = 0; grp[2] < L.ng[2]; grp[2]++)
            for (grp[1] = 0; grp[1] < L.ng[1]; grp[1]++)
                for (grp[0] = 0; grp[0] < L.ng[0]; grp[0]++) {
                    emul_set(&emul_wi, &L, grp, lid);
                    body(args);
                }
        return;
    }
    ucontext_t *ctx = calloc(items, sizeof(*ctx));
    struct emul_item *wi = calloc(items, sizeof(*wi));
    char *stacks = malloc(items * (size_t)EMUL_STACK);
    unsigned char *done = malloc(items);

    launch = &L;
    items_ctx = ctx;
    finished = done;
    for (grp[2] = 0; grp[2] < L.ng[2]; grp[2]++)
        for (grp[1] = 0; grp[1] < L.ng[1]; grp[1]++)
            for (grp[0] = 0; grp[0] < L.ng[0]; grp[0]++) {
                size_t left = items;

                for (size_t i = 0; i < items; i++) {
                    const size_t lid[3] = {i % l[0], i / l[0] % l[1], i / (l[0] * l[1])};

                    emul_set(&wi[i], &L, grp, lid);
                    getcontext(&ctx[i]);
                    ctx[i].uc_stack.ss_sp = stacks + i * (size_t)EMUL_STACK;
                    ctx[i].uc_stack.ss_size = EMUL_STACK;
                    ctx[i].uc_link = &sched;
                    makecontext(&ctx[i], emul_item_main, 0);
                    done[i] = 0;
                }
                in_group = 1;
                /* Round robin: each turn runs a work-item to its next
                 * barrier or to its end. */
                while (left) {
                    for (size_t i = 0; i < items; i++) {
                        if (done[i])
                            continue;
                        current = (int)i;
                        emul_wi = wi[i];
                        swapcontext(&sched, &ctx[i]);
                        wi[i] = emul_wi;
                    }
                    left = 0;
                    for (size_t i = 0; i < items; i++)
                        left += !done[i];
                }
                in_group = 0;
            }
    free(ctx);
    free(wi);
    free(stacks);
    free(done);
}
