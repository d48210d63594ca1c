// SPDX-License-Identifier: Unlicense
//
// The RoMa tile queue (roma_tiles.h): pipelines of backend + ops + model on
// one or more GPUs, one host thread each while a run lasts. A shared
// counter deals the tile indices; each pipeline fills its pinned inputs
// through the caller's get, runs roma_match (one graph launch, copies in
// and out, synchronous), then waits for its turn and hands the results to
// put in index order. A pipeline that finished ahead of an earlier tile
// waits with its results (at most one tile per pipeline is held), so the
// gather needs no extra buffers.

#include <condition_variable>
#include <mutex>
#include <string>
#include <string.h>
#include <thread>
#include <vector>

#include "common.cuh"
#include "pth_loader.h"
#include "roma.h"
#include "roma_tiles.h"

using coreg::cuda_ok;
using coreg::fail;
using coreg::pending;

namespace {

struct Pipe {
    struct ocl_backend ocl;
    struct ops o;
    struct roma_model m;
    float *inA = nullptr, *inB = nullptr;
    bool ready = false;
};

// The error recorded on this thread, taken off it (empty when none).
std::string take_error()
{
    if (!pending())
        return std::string();
    const char *e = coreg_last_error();
    std::string s = e ? e : "unknown error";
    coreg_clear_error();
    return s;
}

// One pipeline's set-up on its own thread: backend, ops, model, buffers.
void pipe_setup(Pipe *p, int dev, int precision, const char *main_w, const char *dino_w,
                const char *v2_w, int H, int W, int coarse, int imagenet, std::string *err)
{
    char opt[16];
    snprintf(opt, sizeof(opt), "%d", dev);
    ocl_init(&p->ocl, opt, nullptr);
    ops_init(&p->o, &p->ocl);
    p->o.precision = precision;
    struct pth_file pf, pd, pv;
    memset(&pf, 0, sizeof(pf));
    memset(&pd, 0, sizeof(pd));
    memset(&pv, 0, sizeof(pv));
    pth_open(&pf, main_w);
    pth_open(&pd, dino_w);
    roma_load(&p->m, &p->o, &pf, &pd);
    pth_close(&pf);
    pth_close(&pd);
    if (v2_w) {
        pth_open(&pv, v2_w);
        roma_load_v2(&p->m, &pv);
        pth_close(&pv);
    }
    p->m.imagenet = imagenet;
    if (coarse != ROMA_COARSE)
        roma_set_coarse(&p->m, coarse);
    roma_alloc(&p->m, H, W);
    const size_t bytes = 3 * (size_t)H * W * sizeof(float);
    if (!pending() && cuda_ok(cudaMallocHost((void **)&p->inA, bytes), "roma_tiles inputs") &&
        cuda_ok(cudaMallocHost((void **)&p->inB, bytes), "roma_tiles inputs"))
        p->ready = true;
    *err = take_error();
}

}  // namespace

struct roma_tiles {
    std::vector<Pipe *> pipes;
    int H, W;
};

extern "C" struct roma_tiles *roma_tiles_create(const int *devices, int ndev, int per_device,
                                                int precision, const char *main_w,
                                                const char *dino_w, const char *v2_w, int H,
                                                int W, int coarse, int imagenet)
{
    if (pending())
        return nullptr;
    if (!devices || ndev < 1 || per_device < 1 || !main_w || !dino_w) {
        fail("roma_tiles_create: %d devices, %d pipelines each", ndev, per_device);
        return nullptr;
    }
    roma_tiles *t = new roma_tiles();
    t->H = H;
    t->W = W;
    const int n = ndev * per_device;
    std::vector<std::string> errs(n);
    std::vector<std::thread> th;
    for (int i = 0; i < n; i++) {
        t->pipes.push_back(new Pipe());
        th.emplace_back(pipe_setup, t->pipes[i], devices[i / per_device], precision, main_w,
                        dino_w, v2_w, H, W, coarse, imagenet, &errs[i]);
    }
    for (auto &x : th)
        x.join();
    for (int i = 0; i < n; i++)
        if (!errs[i].empty() || !t->pipes[i]->ready) {
            std::string e = errs[i].empty() ? "pipeline set-up failed" : errs[i];
            roma_tiles_free(t);
            fail("roma_tiles_create: pipeline %d: %s", i, e.c_str());
            return nullptr;
        }
    return t;
}

extern "C" int roma_tiles_pipelines(const struct roma_tiles *t)
{
    return t ? (int)t->pipes.size() : 0;
}

extern "C" int roma_tiles_run(struct roma_tiles *t, int ntiles, roma_tile_get get,
                              roma_tile_put put, void *ctx)
{
    if (pending())
        return 0;
    if (!t || ntiles < 0 || !get || !put) {
        fail("roma_tiles_run: no queue, callback or tiles (%d)", ntiles);
        return 0;
    }
    std::mutex mu;
    std::condition_variable turn;
    int next = 0, delivered = 0;
    bool stop = false;
    std::string first_error;

    auto worker = [&](Pipe *p) {
        for (;;) {
            int idx;
            {
                std::lock_guard<std::mutex> lk(mu);
                if (stop || next >= ntiles)
                    return;
                idx = next++;
            }
            get(ctx, idx, p->inA, p->inB);
            roma_match(&p->m, p->inA, p->inB, nullptr, idx);
            std::string err = take_error();
            std::unique_lock<std::mutex> lk(mu);
            if (!err.empty()) {
                if (first_error.empty())
                    first_error = "tile " + std::to_string(idx) + ": " + err;
                stop = true;
                turn.notify_all();
                return;
            }
            turn.wait(lk, [&] { return stop || delivered == idx; });
            if (stop)
                return;
            // Callbacks run one at a time, in index order, under the lock.
            put(ctx, idx, p->m.flow, p->m.cert, p->m.v2 ? p->m.sd : nullptr);
            delivered++;
            turn.notify_all();
        }
    };
    std::vector<std::thread> th;
    for (Pipe *p : t->pipes)
        th.emplace_back(worker, p);
    for (auto &x : th)
        x.join();
    if (!first_error.empty())
        fail("roma_tiles_run: %s", first_error.c_str());
    return delivered;
}

extern "C" void roma_tiles_free(struct roma_tiles *t)
{
    if (!t)
        return;
    for (Pipe *p : t->pipes) {
        if (p->ocl.queue) {
            roma_free(&p->m);
            ops_free(&p->o);
            ocl_free(&p->ocl);
        }
        if (p->inA)
            cudaFreeHost(p->inA);
        if (p->inB)
            cudaFreeHost(p->inB);
        delete p;
    }
    delete t;
}
