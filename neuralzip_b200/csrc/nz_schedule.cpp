// Host scheduler of the per-block decode: the runtime's forward pre-hook
// in native code, so that a hook costs one C call.
//
// Replaces the work the reference does in NeuralZipRuntime._decode_block
// (neuralzip/gpu/inference.py:491-493: decode every group of a block on the
// current stream right before the block runs) and adds what the reference
// does not have: decode of whole units of consecutive blocks per launch and
// an overlapped schedule on a side stream with rotating workspace slots.
//
// Unit u decodes into slot u % depth. With overlap, the hook of a unit's
// first block waits for the unit's side-stream decode (or decodes it on the
// compute stream if none is pending) and then starts the side-stream decode
// of the next units of the same forward whose slots are free: a slot is
// free once its previous reader has been enqueued on the compute stream,
// which a "free" event recorded on the compute stream at the current hook
// covers. All ordering between the two streams is by CUDA events; nothing
// here blocks the host.

#include "nz_b200.h"
#include "nz_internal.h"

#include <cuda_runtime.h>

#include <string>
#include <vector>

struct nz_schedule {
    std::vector<nz_launch> launches;  // unit u owns [first[u], first[u + 1])
    std::vector<uint32_t> first;
    std::vector<uint32_t> prev_user;  // previous unit of the same slot (cyclic)
    std::vector<int64_t> resident;    // per slot: unit held or being decoded, -1 unknown
    std::vector<uint8_t> pending;     // per unit: a side-stream decode not yet waited for
    std::vector<cudaEvent_t> free_ev;
    std::vector<cudaEvent_t> done_ev;
    uint32_t n_units = 0;
    uint32_t depth = 1;
    cudaStream_t side = nullptr;
    bool overlap = false;
};

namespace {

int cuda_fail(cudaError_t err, const char* what) {
    return nz::fail(NZ_ECUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

int drain(nz_schedule& s, cudaStream_t stream) {
    for (uint32_t u = 0; u < s.n_units; ++u) {
        if (!s.pending[u]) continue;
        const cudaError_t err = cudaStreamWaitEvent(stream, s.done_ev[u], 0);
        if (err != cudaSuccess) return cuda_fail(err, "cudaStreamWaitEvent");
        s.pending[u] = 0;
    }
    return NZ_OK;
}

int launch_unit(nz_schedule& s, uint32_t unit, cudaStream_t stream) {
    const uint32_t count = s.first[unit + 1] - s.first[unit];
    return nz_decode_launch_many(s.launches.data() + s.first[unit], count, stream);
}

int decode_unit(nz_schedule& s, uint32_t unit, cudaStream_t stream) {
    int rc = drain(s, stream);
    if (rc != NZ_OK) return rc;
    rc = launch_unit(s, unit, stream);
    if (rc != NZ_OK) return rc;
    s.resident[unit % s.depth] = unit;
    return NZ_OK;
}

// Starts the side-stream decode of the units after `unit` in this forward
// (never past the last unit: the next forward's first unit is decoded by
// its own hook, so a forward never relies on workspace contents written
// during the previous one, as the reference decodes each block right
// before it runs).
int prefetch(nz_schedule& s, uint32_t unit, cudaStream_t compute) {
    const uint32_t n = s.n_units;
    bool freed = false;
    for (uint32_t d = 1; d < s.depth && unit + d < n; ++d) {
        const uint32_t next = unit + d;
        if (s.pending[next]) continue;
        // The slot's previous reader must lie before this unit in the
        // enqueue order; one in [unit, next) has not run yet.
        if ((s.prev_user[next] + n - unit) % n < d) break;
        cudaError_t err;
        if (!freed) {
            err = cudaEventRecord(s.free_ev[unit], compute);
            if (err != cudaSuccess) return cuda_fail(err, "cudaEventRecord");
            err = cudaStreamWaitEvent(s.side, s.free_ev[unit], 0);
            if (err != cudaSuccess) return cuda_fail(err, "cudaStreamWaitEvent");
            freed = true;
        }
        const int rc = launch_unit(s, next, s.side);
        if (rc != NZ_OK) return rc;
        err = cudaEventRecord(s.done_ev[next], s.side);
        if (err != cudaSuccess) return cuda_fail(err, "cudaEventRecord");
        s.pending[next] = 1;
        s.resident[next % s.depth] = next;
    }
    return NZ_OK;
}

}  // namespace

extern "C" {

int nz_schedule_create(const nz_launch* launches, const uint32_t* unit_first, uint32_t n_units,
                       uint32_t depth, void* side_stream, nz_schedule** out) {
    NZ_GUARD({
        if (!out || !unit_first || n_units == 0) throw nz::Error(NZ_EVALUE, "Invalid schedule arguments.");
        if (depth == 0) throw nz::Error(NZ_EVALUE, "A schedule needs at least one slot.");
        if (depth > 1 && !side_stream) throw nz::Error(NZ_EVALUE, "An overlapped schedule needs a side stream.");
        const uint32_t total = unit_first[n_units];
        if (unit_first[0] != 0 || (total && !launches))
            throw nz::Error(NZ_EVALUE, "Invalid unit launch ranges.");
        for (uint32_t u = 0; u < n_units; ++u)
            if (unit_first[u] > unit_first[u + 1]) throw nz::Error(NZ_EVALUE, "Invalid unit launch ranges.");
        auto* s = new nz_schedule();
        s->launches.assign(launches, launches + total);
        s->first.assign(unit_first, unit_first + n_units + 1);
        s->n_units = n_units;
        s->depth = depth;
        s->overlap = depth > 1;
        s->side = reinterpret_cast<cudaStream_t>(side_stream);
        s->resident.assign(depth, -1);
        s->pending.assign(n_units, 0);
        s->prev_user.resize(n_units);
        for (uint32_t u = 0; u < n_units; ++u) {
            uint32_t j = (u + n_units - 1) % n_units;
            while (j % depth != u % depth && j != u) j = (j + n_units - 1) % n_units;
            s->prev_user[u] = j;
        }
        if (s->overlap) {
            s->free_ev.assign(n_units, nullptr);
            s->done_ev.assign(n_units, nullptr);
            for (uint32_t u = 0; u < n_units; ++u) {
                cudaError_t err = cudaEventCreateWithFlags(&s->free_ev[u], cudaEventDisableTiming);
                if (err == cudaSuccess) err = cudaEventCreateWithFlags(&s->done_ev[u], cudaEventDisableTiming);
                if (err != cudaSuccess) {
                    nz_schedule_destroy(s);
                    throw nz::Error(NZ_ECUDA, std::string("cudaEventCreate: ") + cudaGetErrorString(err));
                }
            }
        }
        *out = s;
    })
}

int nz_schedule_destroy(nz_schedule* s) {
    if (!s) return NZ_OK;
    for (cudaEvent_t e : s->free_ev)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : s->done_ev)
        if (e) cudaEventDestroy(e);
    delete s;
    return NZ_OK;
}

int nz_schedule_enter(nz_schedule* s, uint32_t unit, uint32_t is_head, void* compute_stream) {
    if (!s || unit >= s->n_units) return nz::fail(NZ_EVALUE, "Invalid schedule unit.");
    cudaStream_t compute = reinterpret_cast<cudaStream_t>(compute_stream);
    const uint32_t slot = unit % s->depth;
    int rc = NZ_OK;
    if (s->pending[unit] && s->resident[slot] == unit) {
        const cudaError_t err = cudaStreamWaitEvent(compute, s->done_ev[unit], 0);
        if (err != cudaSuccess) return cuda_fail(err, "cudaStreamWaitEvent");
        s->pending[unit] = 0;
    } else if (is_head || s->resident[slot] != unit) {
        rc = decode_unit(*s, unit, compute);
        if (rc != NZ_OK) return rc;
    }
    if (is_head && s->overlap) rc = prefetch(*s, unit, compute);
    return rc;
}

int nz_schedule_decode_unit(nz_schedule* s, uint32_t unit, void* stream) {
    if (!s || unit >= s->n_units) return nz::fail(NZ_EVALUE, "Invalid schedule unit.");
    return decode_unit(*s, unit, reinterpret_cast<cudaStream_t>(stream));
}

int nz_schedule_drain(nz_schedule* s, void* stream) {
    if (!s) return nz::fail(NZ_EVALUE, "Null schedule.");
    return drain(*s, reinterpret_cast<cudaStream_t>(stream));
}

int nz_schedule_mark(nz_schedule* s, uint32_t unit, uint32_t whole) {
    if (!s || unit >= s->n_units) return nz::fail(NZ_EVALUE, "Invalid schedule unit.");
    s->resident[unit % s->depth] = whole ? static_cast<int64_t>(unit) : -1;
    return NZ_OK;
}

}  // extern "C"
