// comm.cuh -- the NCCL communicator of libdance_b200 and its bounded waits,
// shared by the sharded standard build and the sharded stitched build.
//
// The communicator is non-blocking (ncclConfig_t.blocking = 0): every host
// wait on it, or on a stream that holds its collectives, polls with a
// deadline; when the deadline passes the communicator is aborted and the
// caller returns -4, so a rank that stops taking part ends the others' calls
// with an error instead of a hang.
#pragma once

#include <nccl.h>

#include <chrono>
#include <thread>

#include "host_common.cuh"

struct DanceComm
{
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
    double timeout_s = 60.0;
    bool aborted = false;
};

namespace dance
{

#define DANCE_NCCL(call)                                                                                      \
    do                                                                                                        \
    {                                                                                                         \
        ncclResult_t r__ = (call);                                                                            \
        if (r__ != ncclSuccess && r__ != ncclInProgress)                                                      \
            return fail(-3, "NCCL error %s at %s:%d (%s)", ncclGetErrorString(r__), __FILE__, __LINE__, #call); \
    } while (0)

using Clock = std::chrono::steady_clock;

// Waits until the communicator has no operation in flight on the host side.
static int nccl_settle(DanceComm *c, Clock::time_point deadline)
{
    while (true)
    {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess)
            return fail(-3, "ncclCommGetAsyncError: %s", ncclGetErrorString(r));
        if (st == ncclSuccess)
            return 0;
        if (st != ncclInProgress)
        {
            ncclCommAbort(c->comm);
            c->aborted = true;
            return fail(-3, "NCCL asynchronous error: %s", ncclGetErrorString(st));
        }
        if (Clock::now() > deadline)
        {
            ncclCommAbort(c->comm);
            c->aborted = true;
            return fail(-4, "NCCL operation did not settle within %.1f s; communicator aborted", c->timeout_s);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Waits for the build stream with the communicator's timeout; a peer that
// stopped participating leaves a collective pending, which ends in an abort.
static int stream_wait(DanceComm *c, cudaStream_t s, Clock::time_point deadline)
{
    while (true)
    {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess)
            return 0;
        if (e != cudaErrorNotReady)
            return fail(-2, "CUDA error %s while waiting for the build stream", cudaGetErrorString(e));
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(c->comm, &st);
        if (st != ncclSuccess && st != ncclInProgress)
        {
            ncclCommAbort(c->comm);
            c->aborted = true;
            return fail(-3, "NCCL asynchronous error: %s", ncclGetErrorString(st));
        }
        if (Clock::now() > deadline)
        {
            ncclCommAbort(c->comm);
            c->aborted = true;
            return fail(-4, "build stream did not finish within %.1f s; communicator aborted", c->timeout_s);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

static Clock::time_point deadline_of(const DanceComm *c)
{
    return Clock::now() + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double>(c->timeout_s));
}

} // namespace dance
