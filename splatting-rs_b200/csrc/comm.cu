// The multi-GPU view-sharded step behind the C ABI: a communicator over NCCL, the exchange of
// the parameter gradients and the Adam step (peer memory, reduce-scatter / all-gather, or
// all-reduce), and the collectives a densification of several ranks needs. With these a caller
// without PyTorch (the reference's Rust `Trainer`, instantsplat-rs/src/training.rs:111-229)
// drives several GPUs through the library alone: sp_comm_unique_id on one rank, the 128 bytes
// passed to the others by any host channel, sp_comm_init on every rank, then per step its
// backward passes and sp_exchange_step.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2: in a process that has already loaded one,
// PyTorch's for example, that one; else the system's), so the library loads, and its
// single-GPU entry points work, where NCCL is absent. The communicator is non-blocking: its
// set-up and every call wait for NCCL on the host only up to the communicator's time limit,
// after which the communicator is aborted and SP_ERR_TIMEOUT returned.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "objects.h"

namespace {

// The NCCL entry points this file uses, looked up once.
struct NcclApi {
    bool loaded = false;
    std::string error;
    int version = 0;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclCommFinalize) finalize = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclReduceScatter) reduce_scatter = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclGetVersion) get_version = nullptr;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            api.error = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown");
            return;
        }
        bool ok = true;
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) {
                ok = false;
                api.error = std::string("libnccl.so.2 lacks ") + name;
            }
        };
        sym(api.get_unique_id, "ncclGetUniqueId");
        sym(api.init_rank_config, "ncclCommInitRankConfig");
        sym(api.finalize, "ncclCommFinalize");
        sym(api.destroy, "ncclCommDestroy");
        sym(api.abort, "ncclCommAbort");
        sym(api.async_error, "ncclCommGetAsyncError");
        sym(api.all_reduce, "ncclAllReduce");
        sym(api.reduce_scatter, "ncclReduceScatter");
        sym(api.all_gather, "ncclAllGather");
        sym(api.error_string, "ncclGetErrorString");
        sym(api.get_version, "ncclGetVersion");
        if (ok) api.get_version(&api.version);
        api.loaded = ok;
    });
    return api;
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct sp_comm {
    sp_context* ctx = nullptr;
    ncclComm_t comm = nullptr;
    uint32_t rank = 0, world = 1;
    uint32_t timeout_ms = 0;
    float* token = nullptr;    // one float: the one-element all-reduce of a barrier
    int32_t* flags = nullptr;  // the agreement of the ranks (an all-reduce of minima)
    bool aborted = false;
};

struct sp_exchange {
    sp_comm* comm = nullptr;
    sp_adam* adam = nullptr;
    uint32_t mode = SP_EXCHANGE_ALLREDUCE;
    sp_peer_exchange* peer = nullptr;
};

namespace {

sp_status nccl_fail(sp_comm* c, ncclResult_t r, const char* what) {
    const char* text = nccl().error_string ? nccl().error_string(r) : "NCCL error";
    return fail(c->ctx, SP_ERR_NCCL, std::string(what) + ": " + text);
}

// Waits on the host until the communicator's pending NCCL call has been taken (its state
// leaves ncclInProgress), up to the time limit; aborts the communicator past it.
sp_status settle(sp_comm* c, ncclResult_t r, const char* what) {
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    while (r == ncclInProgress) {
        if (Clock::now() > deadline) {
            nccl().abort(c->comm);
            c->aborted = true;
            return fail(c->ctx, SP_ERR_TIMEOUT, std::string(what) + ": no answer from every rank within the limit");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
        ncclResult_t state = ncclSuccess;
        const ncclResult_t q = nccl().async_error(c->comm, &state);
        r = q != ncclSuccess ? q : state;
    }
    return r == ncclSuccess ? SP_OK : nccl_fail(c, r, what);
}

#define SP_NCCL(c, expr, what)                                  \
    do {                                                        \
        if ((c)->aborted) return fail((c)->ctx, SP_ERR_NCCL, "the communicator was aborted"); \
        const sp_status s_ = settle((c), (expr), (what));       \
        if (s_ != SP_OK) return s_;                             \
    } while (0)

// A one-element all-reduce on the context's stream: no rank's work enqueued after it runs
// before every rank's work enqueued before it has completed.
sp_status barrier(sp_comm* c) {
    SP_NCCL(c, nccl().all_reduce(c->token, c->token, 1, ncclFloat32, ncclSum, c->comm, c->ctx->stream),
            "barrier all-reduce");
    return SP_OK;
}

// Whether every rank passes `ok`, agreed through an all-reduce of minima (blocks the host).
sp_status agree(sp_comm* c, bool ok, bool* all) {
    const int32_t mine = ok ? 1 : 0;
    SP_CUDA(c->ctx, cudaMemcpyAsync(c->flags, &mine, sizeof(mine), cudaMemcpyHostToDevice, c->ctx->stream));
    SP_NCCL(c, nccl().all_reduce(c->flags, c->flags, 1, ncclInt32, ncclMin, c->comm, c->ctx->stream),
            "agreement all-reduce");
    int32_t every = 0;
    SP_CUDA(c->ctx, cudaMemcpyAsync(&every, c->flags, sizeof(every), cudaMemcpyDeviceToHost, c->ctx->stream));
    SP_CHECK(sync_stream(c->ctx));
    *all = every == 1;
    return SP_OK;
}

}  // namespace

extern "C" {

sp_status sp_comm_unique_id(uint8_t out[SP_COMM_ID_BYTES]) {
    if (!out) return SP_ERR_INVALID;
    NcclApi& api = nccl();
    if (!api.loaded) return SP_ERR_NCCL;
    static_assert(sizeof(ncclUniqueId) == SP_COMM_ID_BYTES, "NCCL's unique id is 128 bytes");
    ncclUniqueId id;
    if (api.get_unique_id(&id) != ncclSuccess) return SP_ERR_NCCL;
    std::memcpy(out, &id, sizeof(id));
    return SP_OK;
}

int sp_comm_nccl_version(void) { return nccl().loaded ? nccl().version : 0; }

sp_status sp_comm_init(sp_context* ctx, const uint8_t id[SP_COMM_ID_BYTES], uint32_t world, uint32_t rank,
                       uint32_t timeout_ms, sp_comm** out) {
    if (!ctx || !id || !out) return SP_ERR_INVALID;
    *out = nullptr;
    SP_REQUIRE(ctx, world >= 1 && rank < world, SP_ERR_INVALID, "rank outside the world");
    SP_REQUIRE(ctx, timeout_ms > 0, SP_ERR_INVALID, "a time limit is required");
    NcclApi& api = nccl();
    if (!api.loaded) return fail(ctx, SP_ERR_NCCL, api.error);
    SP_CHECK(select_device(ctx));
    sp_comm* c = new sp_comm();
    c->ctx = ctx;
    c->rank = rank;
    c->world = world;
    c->timeout_ms = timeout_ms;
    cudaError_t err = cudaMalloc(&c->token, sizeof(float));
    if (err == cudaSuccess) err = cudaMemset(c->token, 0, sizeof(float));
    if (err == cudaSuccess) err = cudaMalloc(&c->flags, sizeof(int32_t));
    if (err != cudaSuccess) {
        cudaFree(c->token);
        cudaFree(c->flags);
        delete c;
        return cuda_fail(ctx, err, "communicator buffers");
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    const ncclResult_t r = api.init_rank_config(&c->comm, (int)world, uid, (int)rank, &config);
    sp_status s = c->comm ? settle(c, r, "ncclCommInitRankConfig") : nccl_fail(c, r, "ncclCommInitRankConfig");
    if (s != SP_OK) {
        if (c->comm && !c->aborted) api.abort(c->comm);
        cudaFree(c->token);
        cudaFree(c->flags);
        delete c;
        return s;
    }
    *out = c;
    return SP_OK;
}

void sp_comm_destroy(sp_comm* c) {
    if (!c) return;
    cudaSetDevice(c->ctx->device);
    if (c->comm && !c->aborted) {
        cudaStreamSynchronize(c->ctx->stream);
        // Finalize (flushes the communicator's work), then free it; abort if it does not settle.
        if (settle(c, nccl().finalize(c->comm), "ncclCommFinalize") == SP_OK) nccl().destroy(c->comm);
        else if (!c->aborted) nccl().abort(c->comm);
    }
    cudaFree(c->token);
    cudaFree(c->flags);
    delete c;
}

uint32_t sp_comm_rank(const sp_comm* c) { return c ? c->rank : 0; }

uint32_t sp_comm_world(const sp_comm* c) { return c ? c->world : 0; }

sp_status sp_comm_barrier(sp_comm* c) {
    if (!c) return SP_ERR_INVALID;
    SP_CHECK(select_device(c->ctx));
    return barrier(c);
}

sp_status sp_comm_wait(sp_comm* c) {
    if (!c) return SP_ERR_INVALID;
    SP_CHECK(select_device(c->ctx));
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(c->ctx->stream);
        if (q == cudaSuccess) return SP_OK;
        if (q != cudaErrorNotReady) return cuda_fail(c->ctx, q, "cudaStreamQuery");
        ncclResult_t state = ncclSuccess;
        if (!c->aborted && nccl().async_error(c->comm, &state) == ncclSuccess && state != ncclSuccess &&
            state != ncclInProgress) {
            nccl().abort(c->comm);
            c->aborted = true;
            return nccl_fail(c, state, "a collective failed");
        }
        if (Clock::now() > deadline) {
            if (!c->aborted) nccl().abort(c->comm);
            c->aborted = true;
            return fail(c->ctx, SP_ERR_TIMEOUT, "the context's stream did not finish within the limit");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

sp_status sp_allreduce_grads(sp_comm* c, sp_rasterizer* r) {
    if (!c || !r || r->ctx != c->ctx) return SP_ERR_INVALID;
    SP_CHECK(select_device(c->ctx));
    SP_NCCL(c, nccl().all_reduce(r->param_gradients, r->param_gradients, r->n * r->stride, ncclFloat32, ncclSum,
                                 c->comm, c->ctx->stream),
            "gradient all-reduce");
    return SP_OK;
}

sp_status sp_adam_step_sharded(sp_comm* c, sp_adam* a, float position_rate_factor) {
    if (!c || !a || a->ctx != c->ctx) return SP_ERR_INVALID;
    SP_REQUIRE(c->ctx, a->n % c->world == 0, SP_ERR_INVALID, "the Gaussians do not split evenly over the ranks");
    SP_CHECK(select_device(c->ctx));
    const uint64_t share = a->n / c->world, floats = share * a->stride;
    float* gradients = const_cast<float*>(a->gradients);
    // In place: this rank's share of the gradient buffer receives the sum over the ranks.
    SP_NCCL(c, nccl().reduce_scatter(gradients, gradients + c->rank * floats, floats, ncclFloat32, ncclSum, c->comm,
                                     c->ctx->stream),
            "gradient reduce-scatter");
    SP_CHECK(sp_adam_advance(a, position_rate_factor));
    SP_CHECK(sp_adam_step_range(a, c->rank * share, share));
    SP_NCCL(c, nccl().all_gather(a->params + c->rank * floats, a->params, floats, ncclFloat32, c->comm,
                                 c->ctx->stream),
            "parameter all-gather");
    return SP_OK;
}

sp_status sp_exchange_create(sp_comm* c, sp_adam* a, uint32_t mode, sp_exchange** out) {
    if (!c || !a || !out || a->ctx != c->ctx) return SP_ERR_INVALID;
    *out = nullptr;
    SP_REQUIRE(c->ctx, mode <= SP_EXCHANGE_ALLREDUCE, SP_ERR_INVALID, "exchange mode");
    SP_CHECK(select_device(c->ctx));
    const bool even = a->n % c->world == 0;
    SP_REQUIRE(c->ctx, even || mode == SP_EXCHANGE_AUTO || mode == SP_EXCHANGE_ALLREDUCE, SP_ERR_INVALID,
               "the Gaussians do not split evenly over the ranks");
    sp_exchange* ex = new sp_exchange();
    ex->comm = c;
    ex->adam = a;
    ex->mode = mode == SP_EXCHANGE_AUTO ? (even ? SP_EXCHANGE_PEER : SP_EXCHANGE_ALLREDUCE) : mode;
    if (ex->mode == SP_EXCHANGE_PEER && c->world > 1) {
        // Every rank exports its buffers, the handles are all-gathered, every rank maps its
        // peers', and the ranks agree that all of them could; every rank takes each of these
        // steps, whatever failed, so that the collectives match.
        sp_peer_handle own{};
        const bool exported = sp_peer_export(a, &own) == SP_OK;
        std::vector<sp_peer_handle> handles(c->world);
        sp_peer_handle* d_handles = nullptr;
        SP_CUDA(c->ctx, cudaMalloc(&d_handles, sizeof(sp_peer_handle) * c->world));
        cudaError_t err = cudaMemcpyAsync(d_handles + c->rank, &own, sizeof(own), cudaMemcpyHostToDevice,
                                          c->ctx->stream);
        sp_status s = err == cudaSuccess ? SP_OK : cuda_fail(c->ctx, err, "handle upload");
        if (s == SP_OK)
            s = settle(c,
                       nccl().all_gather(d_handles + c->rank, d_handles, sizeof(sp_peer_handle), ncclUint8, c->comm,
                                         c->ctx->stream),
                       "handle all-gather");
        if (s == SP_OK) {
            err = cudaMemcpyAsync(handles.data(), d_handles, sizeof(sp_peer_handle) * c->world,
                                  cudaMemcpyDeviceToHost, c->ctx->stream);
            s = err == cudaSuccess ? sync_stream(c->ctx) : cuda_fail(c->ctx, err, "handle download");
        }
        cudaFree(d_handles);
        if (s != SP_OK) {
            delete ex;
            return s;
        }
        bool mapped = false;
        if (exported) {
            bool complete = true;
            for (const sp_peer_handle& h : handles) complete = complete && h.gaussian_count == a->n;
            mapped = complete && sp_peer_exchange_create(a, c->rank, c->world, handles.data(), &ex->peer) == SP_OK;
        }
        bool all = false;
        s = agree(c, mapped, &all);
        if (s != SP_OK || !all) {
            sp_peer_exchange_destroy(ex->peer);
            ex->peer = nullptr;
            if (s != SP_OK || mode == SP_EXCHANGE_PEER) {
                delete ex;
                return s != SP_OK ? s : fail(c->ctx, SP_ERR_CUDA, "a rank could not map its peers' buffers");
            }
            ex->mode = SP_EXCHANGE_SHARDED;  // the collective form, the same bytes over NVLink
        }
    }
    *out = ex;
    return SP_OK;
}

uint32_t sp_exchange_mode(const sp_exchange* ex) { return ex ? ex->mode : 0; }

sp_status sp_exchange_probe_link(sp_exchange* ex, uint32_t peer, uint64_t bytes, float* milliseconds) {
    if (!ex || !milliseconds) return SP_ERR_INVALID;
    sp_comm* c = ex->comm;
    SP_REQUIRE(c->ctx, ex->peer != nullptr, SP_ERR_INVALID, "the exchange does not use peer memory");
    SP_REQUIRE(c->ctx, peer < c->world && peer != c->rank, SP_ERR_INVALID, "the peer must be another rank");
    const sp_adam* a = ex->adam;
    SP_REQUIRE(c->ctx, bytes > 0 && bytes % 16 == 0 && bytes <= a->n * a->stride * sizeof(float), SP_ERR_INVALID,
               "bytes: a multiple of 16 within the peer's gradient buffer");
    SP_CHECK(select_device(c->ctx));
    const float4* src = reinterpret_cast<const float4*>(ex->peer->peers.gradients[peer]);
    SP_REQUIRE(c->ctx, (reinterpret_cast<uintptr_t>(src) & 15u) == 0, SP_ERR_INVALID, "unaligned peer buffer");
    int sms = 0;
    SP_CUDA(c->ctx, cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->ctx->device));
    const unsigned blocks = (unsigned)std::max(sms, 1) * 4u;
    float4* sink = nullptr;
    SP_CUDA(c->ctx, cudaMalloc(&sink, blocks * sizeof(float4)));
    cudaEvent_t start = nullptr, stop = nullptr;
    cudaEventCreate(&start);
    cudaEventCreate(&stop);
    cudaStream_t st = c->ctx->stream;
    // One untimed pass (maps the pages), then the timed one.
    cudaError_t err = splat::launch_peer_read(src, bytes / 16, sink, blocks, st);
    if (err == cudaSuccess) err = cudaEventRecord(start, st);
    if (err == cudaSuccess) err = splat::launch_peer_read(src, bytes / 16, sink, blocks, st);
    if (err == cudaSuccess) err = cudaEventRecord(stop, st);
    if (err == cudaSuccess) err = cudaEventSynchronize(stop);
    if (err == cudaSuccess) err = cudaEventElapsedTime(milliseconds, start, stop);
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    cudaFree(sink);
    return err == cudaSuccess ? SP_OK : cuda_fail(c->ctx, err, "peer-read probe");
}

sp_status sp_exchange_step(sp_exchange* ex, float position_rate_factor) {
    NvtxRange range("sp_exchange_step");
    if (!ex) return SP_ERR_INVALID;
    sp_comm* c = ex->comm;
    SP_CHECK(select_device(c->ctx));
    if (c->world == 1) return sp_adam_step(ex->adam, position_rate_factor);
    switch (ex->mode) {
        case SP_EXCHANGE_PEER:
            SP_CHECK(barrier(c));  // every rank's gradients are written
            SP_CHECK(sp_peer_exchange_step(ex->peer, position_rate_factor));
            return barrier(c);     // every rank's parameters are written
        case SP_EXCHANGE_SHARDED:
            return sp_adam_step_sharded(c, ex->adam, position_rate_factor);
        default: {
            sp_adam* a = ex->adam;
            float* gradients = const_cast<float*>(a->gradients);
            SP_NCCL(c, nccl().all_reduce(gradients, gradients, a->n * a->stride, ncclFloat32, ncclSum, c->comm,
                                         c->ctx->stream),
                    "gradient all-reduce");
            return sp_adam_step(a, position_rate_factor);
        }
    }
}

sp_status sp_exchange_gather_moments(sp_exchange* ex) {
    if (!ex) return SP_ERR_INVALID;
    sp_comm* c = ex->comm;
    if (c->world == 1 || ex->mode == SP_EXCHANGE_ALLREDUCE) return SP_OK;
    SP_CHECK(select_device(c->ctx));
    sp_adam* a = ex->adam;
    const uint64_t floats = a->n / c->world * a->stride;
    for (float* m : {a->first_moment, a->second_moment})
        SP_NCCL(c, nccl().all_gather(m + c->rank * floats, m, floats, ncclFloat32, c->comm, c->ctx->stream),
                "moment all-gather");
    return SP_OK;
}

void sp_exchange_destroy(sp_exchange* ex) {
    if (!ex) return;
    sp_peer_exchange_destroy(ex->peer);
    delete ex;
}

sp_status sp_comm_merge_densify_stats(sp_comm* c, sp_rasterizer* r) {
    if (!c || !r || r->ctx != c->ctx) return SP_ERR_INVALID;
    if (c->world == 1) return SP_OK;
    SP_CHECK(select_device(c->ctx));
    float4* summed = nullptr;
    SP_CUDA(c->ctx, cudaMalloc(&summed, r->n * sizeof(float4)));
    cudaStream_t st = c->ctx->stream;
    cudaError_t err = cudaMemcpyAsync(summed, r->densify_stats, r->n * sizeof(float4), cudaMemcpyDeviceToDevice, st);
    sp_status s = err == cudaSuccess ? SP_OK : cuda_fail(c->ctx, err, "statistics copy");
    // The mean-gradient sums and visible counts summed, the largest screen radius kept.
    if (s == SP_OK)
        s = settle(c, nccl().all_reduce(summed, summed, r->n * 4, ncclFloat32, ncclSum, c->comm, st),
                   "statistics all-reduce (sum)");
    if (s == SP_OK)
        s = settle(c,
                   nccl().all_reduce(r->densify_stats, r->densify_stats, r->n * 4, ncclFloat32, ncclMax, c->comm, st),
                   "statistics all-reduce (max)");
    if (s == SP_OK) {
        err = cudaMemcpy2DAsync(r->densify_stats, sizeof(float4), summed, sizeof(float4), 2 * sizeof(float), r->n,
                                cudaMemcpyDeviceToDevice, st);
        s = err == cudaSuccess ? sync_stream(c->ctx) : cuda_fail(c->ctx, err, "statistics merge");
    }
    cudaFree(summed);
    return s;
}

}  // extern "C"
