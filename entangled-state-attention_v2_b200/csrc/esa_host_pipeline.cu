// esa_host_pipeline.cu -- forward scan of HOST-resident A, B into host E,
// with the host<->device copies pipelined against the scan.
//
// The tensor is cut into contiguous chunks of about 32 MB per array (whole
// batch rows when a row is small, else time pieces of one row, chained
// through the acc-type end state e_last -> e0).  Chunk i goes through three
// queues:
//
//   copy-in stream : A_i, B_i host -> staging slot (i mod the slot count)
//   caller stream  : scan of slot i (esa_scan_fwd on the device copies)
//   copy-out stream: E_i staging slot -> host
//
// so the host->device copy of chunk i+1, the scan of chunk i and the
// device->host copy of chunk i-1 run at the same time (PCIe is full duplex
// and the copy engines are separate from the SMs).  A slot is refilled only
// after its previous scan finished reading it and its previous E was copied
// out; the events that express this are reused per slot (cudaStreamWaitEvent
// waits for the latest record made before the call).  The library still
// allocates nothing: the staging slots, the scan workspace and the chunk
// carries live in the caller's `staging` buffer.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "../../include/esa_b200.h"
#include "esa_internal.h"

namespace esa {
namespace {

constexpr int kMaxSlots = 8;

// staging slots per array (more than 3 gained nothing)
int slots() { return 3; }
int64_t chunk_bytes() {
    // 32 MB: measured 70 GB/s end to end on [32,4096,16,64] fp16 against 65 at
    // 8 MB (per-copy overheads); more slots than 3 gained nothing
    return (int64_t)32 << 20;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Plan {
    int64_t rows_per_chunk;   // batch rows per chunk
    int64_t steps_per_chunk;  // time steps per chunk (== T when rows are whole)
    int64_t pieces_per_row;   // time pieces per row (1 when rows are whole)
    int64_t nchunks;
    size_t slot_array_bytes;  // bytes of one array of one slot
    size_t ws_bytes;          // scan workspace for the largest chunk
    size_t carry_bytes;       // one [hd] acc-type state
    size_t total;
};

Plan make_plan(int64_t nb, int64_t T, int64_t hd, int es, int compass) {
    Plan p{};
    const int64_t row_bytes = T * hd * es;
    const int64_t chunk = chunk_bytes();
    if (row_bytes <= chunk) {
        p.rows_per_chunk = row_bytes > 0 ? std::max<int64_t>(1, chunk / row_bytes) : 1;
        p.rows_per_chunk = std::min<int64_t>(p.rows_per_chunk, std::max<int64_t>(nb, 1));
        p.steps_per_chunk = T;
        p.pieces_per_row = 1;
        p.nchunks = (nb + p.rows_per_chunk - 1) / p.rows_per_chunk;
    } else {
        p.rows_per_chunk = 1;
        p.steps_per_chunk = std::max<int64_t>(1, chunk / (hd * es));
        p.pieces_per_row = (T + p.steps_per_chunk - 1) / p.steps_per_chunk;
        p.nchunks = nb * p.pieces_per_row;
    }
    const int acc_es = es == 8 ? 8 : 4;
    p.slot_array_bytes = round_up(size_t(p.rows_per_chunk) * p.steps_per_chunk * hd * es, 256);
    p.ws_bytes = round_up(scan_workspace_bytes(p.rows_per_chunk, p.steps_per_chunk, hd, es, compass), 256);
    p.carry_bytes = round_up(size_t(hd) * acc_es, 256);
    p.total = size_t(slots()) * 3 * p.slot_array_bytes + p.ws_bytes + 2 * p.carry_bytes;
    return p;
}

// copy streams and events, created once per device
struct DeviceQueues {
    bool ready = false;
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t start = nullptr, end = nullptr;
    cudaEvent_t loaded[kMaxSlots], scanned[kMaxSlots], stored[kMaxSlots];
};

std::mutex g_mu;
DeviceQueues g_queues[64];

int queues_for(int dev, DeviceQueues** q) {
    if (dev < 0 || dev >= 64) return set_error(ESA_ERR_CUDA, "device ordinal out of range");
    DeviceQueues& d = g_queues[dev];
    if (!d.ready) {
        bool ok = cudaStreamCreateWithFlags(&d.in, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&d.out, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&d.start, cudaEventDisableTiming) == cudaSuccess &&
                  cudaEventCreateWithFlags(&d.end, cudaEventDisableTiming) == cudaSuccess;
        for (int k = 0; ok && k < kMaxSlots; ++k)
            ok = cudaEventCreateWithFlags(&d.loaded[k], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&d.scanned[k], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&d.stored[k], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) return set_error(ESA_ERR_CUDA, "cannot create the copy streams");
        d.ready = true;
    }
    *q = &d;
    return ESA_OK;
}

}  // namespace

size_t scan_host_staging_bytes(int64_t nb, int64_t T, int64_t hd, int es, int compass) {
    return make_plan(nb, T, hd, es, compass).total;
}

int scan_fwd_host(const void* A, const void* B, void* E, int64_t nb, int64_t T, int64_t hd, int dtype,
                  int compass, void* staging, size_t staging_bytes, cudaStream_t s) {
    if (nb < 0 || T < 0 || hd < 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "negative dimension");
    if (compass <= 0) return set_error(ESA_ERR_INVALID_ARGUMENT, "compass must be a positive integer");
    const int es = dtype_size(dtype);
    if (es == 0) return set_error(ESA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code " + std::to_string(dtype));
    if (nb * T * hd == 0) return ESA_OK;
    if (!A || !B || !E) return set_error(ESA_ERR_INVALID_ARGUMENT, "null host pointer");
    const Plan p = make_plan(nb, T, hd, es, compass);
    if (staging == nullptr || staging_bytes < p.total)
        return set_error(ESA_ERR_WORKSPACE, "staging buffer smaller than esa_scan_host_staging_bytes (" +
                                                std::to_string(p.total) + " bytes)");
    if (reinterpret_cast<uintptr_t>(staging) % 256 != 0)
        return set_error(ESA_ERR_INVALID_ARGUMENT, "staging buffer must be 256-byte aligned");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_error(ESA_ERR_CUDA, "cudaGetDevice failed");
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceQueues* q = nullptr;
    if (int rc = queues_for(dev, &q)) return rc;

    const int nslot = slots();
    char* base = static_cast<char*>(staging);
    char* slot[kMaxSlots][3];
    for (int k = 0; k < nslot; ++k)
        for (int a = 0; a < 3; ++a) slot[k][a] = base + (size_t(k) * 3 + a) * p.slot_array_bytes;
    char* ws = base + size_t(nslot) * 3 * p.slot_array_bytes;
    char* carry[2] = {ws + p.ws_bytes, ws + p.ws_bytes + p.carry_bytes};

    const char* hA = static_cast<const char*>(A);
    const char* hB = static_cast<const char*>(B);
    char* hE = static_cast<char*>(E);
    int rc = ESA_OK;
    auto cuda_ok = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && rc == ESA_OK)
            rc = set_error(ESA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
        return rc == ESA_OK;
    };

    // everything the caller queued on `s` before this call comes first
    cuda_ok(cudaEventRecord(q->start, s), "cudaEventRecord");
    cuda_ok(cudaStreamWaitEvent(q->in, q->start, 0), "cudaStreamWaitEvent");
    cuda_ok(cudaStreamWaitEvent(q->out, q->start, 0), "cudaStreamWaitEvent");

    for (int64_t i = 0; i < p.nchunks && rc == ESA_OK; ++i) {
        const int k = int(i % nslot);
        int64_t r0, nr, t0, nt;
        if (p.pieces_per_row == 1) {
            r0 = i * p.rows_per_chunk;
            nr = std::min(p.rows_per_chunk, nb - r0);
            t0 = 0;
            nt = T;
        } else {
            r0 = i / p.pieces_per_row;
            nr = 1;
            t0 = (i % p.pieces_per_row) * p.steps_per_chunk;
            nt = std::min(p.steps_per_chunk, T - t0);
        }
        const size_t off = size_t((r0 * T + t0) * hd) * es;
        const size_t bytes = size_t(nr * nt * hd) * es;
        // copy in, once the scan of chunk i - nslot has finished reading the slot
        if (i >= nslot) cuda_ok(cudaStreamWaitEvent(q->in, q->scanned[k], 0), "cudaStreamWaitEvent");
        cuda_ok(cudaMemcpyAsync(slot[k][0], hA + off, bytes, cudaMemcpyHostToDevice, q->in), "copy of A");
        cuda_ok(cudaMemcpyAsync(slot[k][1], hB + off, bytes, cudaMemcpyHostToDevice, q->in), "copy of B");
        cuda_ok(cudaEventRecord(q->loaded[k], q->in), "cudaEventRecord");
        // scan, once the inputs are in and E of chunk i - nslot has left the slot
        cuda_ok(cudaStreamWaitEvent(s, q->loaded[k], 0), "cudaStreamWaitEvent");
        if (i >= nslot) cuda_ok(cudaStreamWaitEvent(s, q->stored[k], 0), "cudaStreamWaitEvent");
        if (rc != ESA_OK) break;
        const int64_t piece = p.pieces_per_row == 1 ? 0 : i % p.pieces_per_row;
        const void* e0 = piece > 0 ? carry[(piece - 1) & 1] : nullptr;
        void* e_last = (p.pieces_per_row > 1 && piece + 1 < p.pieces_per_row) ? carry[piece & 1] : nullptr;
        rc = scan_fwd(slot[k][0], slot[k][1], slot[k][2], nr, nt, hd, dtype, compass, e0, e_last, ws,
                      p.ws_bytes, s);
        if (rc != ESA_OK) break;
        cuda_ok(cudaEventRecord(q->scanned[k], s), "cudaEventRecord");
        // copy out
        cuda_ok(cudaStreamWaitEvent(q->out, q->scanned[k], 0), "cudaStreamWaitEvent");
        cuda_ok(cudaMemcpyAsync(hE + off, slot[k][2], bytes, cudaMemcpyDeviceToHost, q->out), "copy of E");
        cuda_ok(cudaEventRecord(q->stored[k], q->out), "cudaEventRecord");
    }
    // work queued on `s` after this call sees every copy finished (also on error,
    // so that no copy still reads or writes the caller's buffers unseen)
    const int rc_body = rc;
    rc = ESA_OK;
    cuda_ok(cudaEventRecord(q->end, q->in), "cudaEventRecord");
    cuda_ok(cudaStreamWaitEvent(q->out, q->end, 0), "cudaStreamWaitEvent");
    cuda_ok(cudaEventRecord(q->end, q->out), "cudaEventRecord");
    cuda_ok(cudaStreamWaitEvent(s, q->end, 0), "cudaStreamWaitEvent");
    return rc_body != ESA_OK ? rc_body : rc;
}

}  // namespace esa
