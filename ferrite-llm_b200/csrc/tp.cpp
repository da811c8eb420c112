// Tensor-parallel exchange regions (fb_comm_*): one device region per rank,
// mapped into every rank's process with CUDA IPC so that kernels store
// partial sums (tagged with the exchange's sequence number) straight into
// peers' memory over NVLink.
//
// The reference has no tensor parallelism; its multi-GPU layer enables peer
// access and reduces with peer copies gathered to a root device
// (ferrite-os/native/core/runtime/modules/hot_multi_gpu_primitives.inl:99-123,
// hot_multi_gpu_reduction.inl).  Here every rank pushes its row-parallel
// partials to all ranks from the projection kernel itself, so no copy or
// collective launch sits between the projection and the next norm.
#include <string.h>

#include <memory>

#include "fb_internal.h"

namespace fb {

static size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

CommLayout comm_layout(int world, int max_batch, int hidden) {
    CommLayout L{};
    size_t off = 0;
    L.flags = off;
    off += up256((size_t)FB_TP_MAX * 4);
    L.am_flags = off;
    off += up256((size_t)FB_TP_MAX * max_batch * 4);
    L.inbox_o = off;
    off += up256((size_t)world * max_batch * hidden * 16);
    L.inbox_d = off;
    off += up256((size_t)world * max_batch * hidden * 16);
    L.am_inbox = off;
    off += up256((size_t)world * max_batch * 8);
    L.total = off;
    return L;
}

}  // namespace fb

using namespace fb;

fb_comm::~fb_comm() {
    if (opened)
        for (int p = 0; p < world; p++)
            if (p != rank && peer[p]) cudaIpcCloseMemHandle(peer[p]);
}

extern "C" {

int fb_comm_create(fb_ctx *ctx, int rank, int world, int max_batch, int hidden, fb_comm **out) {
    return guarded([&] {
        FB_REQUIRE(ctx && out, "null argument");
        *out = nullptr;
        FB_REQUIRE(world == 2 || world == 4 || world == 8, "world must be 2, 4 or 8");
        FB_REQUIRE(rank >= 0 && rank < world, "rank out of range");
        FB_REQUIRE(max_batch >= 1 && max_batch <= 32 && hidden > 0 && hidden % 256 == 0,
                   "need 1 <= max_batch <= 32 and hidden a multiple of 256");
        static_assert(sizeof(cudaIpcMemHandle_t) == FB_COMM_HANDLE_BYTES, "IPC handle size");
        FB_CUDA(cudaSetDevice(ctx->device));
        auto c = std::make_unique<fb_comm>();
        c->ctx = ctx;
        c->rank = rank;
        c->world = world;
        c->max_batch = max_batch;
        c->hidden = hidden;
        c->L = comm_layout(world, max_batch, hidden);
        c->region.alloc(c->L.total);  // cudaMalloc: exportable through IPC
        FB_CUDA(cudaMemset(c->region.ptr, 0, c->L.total));
        c->peer[rank] = c->region.as<uint8_t>();
        *out = c.release();
    });
}

int fb_comm_handle(const fb_comm *comm, void *handle_out) {
    return guarded([&] {
        FB_REQUIRE(comm && handle_out, "null argument");
        cudaIpcMemHandle_t h;
        FB_CUDA(cudaIpcGetMemHandle(&h, comm->region.ptr));
        memcpy(handle_out, &h, sizeof(h));
    });
}

int fb_comm_open(fb_comm *comm, const void *handles) {
    return guarded([&] {
        FB_REQUIRE(comm && handles, "null argument");
        FB_REQUIRE(!comm->opened, "comm already opened");
        FB_CUDA(cudaSetDevice(comm->ctx->device));
        const uint8_t *hb = static_cast<const uint8_t *>(handles);
        int opened_upto = 0;
        try {
            for (int p = 0; p < comm->world; p++, opened_upto = p) {
                if (p == comm->rank) continue;
                cudaIpcMemHandle_t h;
                memcpy(&h, hb + (size_t)p * FB_COMM_HANDLE_BYTES, sizeof(h));
                void *ptr = nullptr;
                FB_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
                comm->peer[p] = static_cast<uint8_t *>(ptr);
            }
        } catch (...) {
            for (int p = 0; p < opened_upto; p++)
                if (p != comm->rank && comm->peer[p]) {
                    cudaIpcCloseMemHandle(comm->peer[p]);
                    comm->peer[p] = nullptr;
                }
            throw;
        }
        comm->opened = true;
    });
}

int fb_comm_set_timeout_ms(fb_comm *comm, int ms) {
    return guarded([&] {
        FB_REQUIRE(comm && ms >= 1 && ms <= 600000, "timeout must be 1 ms .. 10 min");
        comm->timeout_ns = (uint64_t)ms * 1000000ull;
    });
}

int fb_comm_destroy(fb_comm *comm) {
    return guarded([&] {
        if (!comm) return;
        cudaSetDevice(comm->ctx->device);
        cudaDeviceSynchronize();
        delete comm;
    });
}

}  // extern "C"
