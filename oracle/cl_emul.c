/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the work-group runner of cl_emul.h. A launch with
 * one work-item per group runs its items in order on the calling thread;
 * a launch with L > 1 items per group starts L threads, which walk the
 * groups in order together, meeting at a barrier after each group (so
 * that the group's local statics can be reused) and wherever the kernel
 * calls barrier(). */

#include <pthread.h>
#include <stdlib.h>

#include "cl_emul.h"

__thread struct emul_item emul_wi;

static pthread_barrier_t group_barrier;
static int group_of_one;

void emul_barrier(void)
{
    if (!group_of_one)
        pthread_barrier_wait(&group_barrier);
}

struct emul_launch {
    void (*body)(void *);
    void *args;
    size_t g[3], l[3], ng[3];
};

struct emul_thread {
    const struct emul_launch *launch;
    size_t lid[3];
    pthread_t th;
};

static void emul_set(const struct emul_launch *L, const size_t grp[3], const size_t lid[3])
{
    for (int d = 0; d < 3; d++) {
        emul_wi.grp[d] = grp[d];
        emul_wi.lid[d] = lid[d];
        emul_wi.gid[d] = grp[d] * L->l[d] + lid[d];
        emul_wi.lsz[d] = L->l[d];
        emul_wi.gsz[d] = L->g[d];
    }
}

static void *emul_worker(void *p)
{
    struct emul_thread *t = p;
    const struct emul_launch *L = t->launch;
    size_t grp[3];

    for (grp[2] = 0; grp[2] < L->ng[2]; grp[2]++)
        for (grp[1] = 0; grp[1] < L->ng[1]; grp[1]++)
            for (grp[0] = 0; grp[0] < L->ng[0]; grp[0]++) {
                emul_set(L, grp, t->lid);
                L->body(L->args);
                pthread_barrier_wait(&group_barrier);
            }
    return NULL;
}

void emul_launch(void (*body)(void *), void *args, const size_t g[3], const size_t l[3])
{
    struct emul_launch L;
    size_t items = 1;

    L.body = body;
    L.args = args;
    for (int d = 0; d < 3; d++) {
        L.g[d] = g[d];
        L.l[d] = l[d];
        L.ng[d] = g[d] / l[d];
        items *= l[d];
    }
    group_of_one = items == 1;
    if (items == 1) {
        size_t grp[3], lid[3] = {0, 0, 0};

        for (grp[2] = 0; grp[2] < L.ng[2]; grp[2]++)
            for (grp[1] = 0; grp[1] < L.ng[1]; grp[1]++)
                for (grp[0] = 0; grp[0] < L.ng[0]; grp[0]++) {
                    emul_set(&L, grp, lid);
                    body(args);
                }
        return;
    }
    struct emul_thread *th = calloc(items, sizeof(*th));
    pthread_barrier_init(&group_barrier, NULL, (unsigned)items);
    for (size_t i = 0; i < items; i++) {
        th[i].launch = &L;
        th[i].lid[0] = i % l[0];
        th[i].lid[1] = i / l[0] % l[1];
        th[i].lid[2] = i / (l[0] * l[1]);
        pthread_create(&th[i].th, NULL, emul_worker, &th[i]);
    }
    for (size_t i = 0; i < items; i++)
        pthread_join(th[i].th, NULL);
    pthread_barrier_destroy(&group_barrier);
    free(th);
}
