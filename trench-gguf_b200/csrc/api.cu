// api.cu - the C ABI of libgpuq_cuda.so (include/gpuq.h): trench-gguf's 12 entry points with the same signatures,
// argument meaning and return conventions (gpuq.hip:2059-2328), plus extensions found by the callers through
// hasattr (gpuq_last_error, gpuq_status, gpuq_init_devices, gpuq_device_count).
//
// Host API (gpuq_quantize*, gpuq_requantize*): host pointers in, host bytes out, synchronous like the reference,
// but internally a pipeline: the blocks are cut into chunks (whole matrices, or row ranges of one big matrix);
// chunk k+1's host-to-device copy, chunk k's kernel and chunk k-1's device-to-host copy run at the same time on
// three streams with two device buffers each. The source bytes are decoded inside the quantize kernel (no float32
// copy in HBM). With several devices (gpuq_init_devices) the chunks are dealt to one host thread a device.
// Device API (gpuq_*_dev): device pointers, the caller's stream, no synchronisation, no library scratch.
#include <algorithm>
#include <cstdarg>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>
#include "common.cuh"
#include "kernels.h"
#include "../../include/gpuq.h"

namespace gq {
namespace {

thread_local std::string t_err;
void set_err(const char * fmt, ...) __attribute__((format(printf, 1, 2)));
void set_err(const char * fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_err = buf;
}

// ------------------------------------------------------------------------------------------------ tables (host)
struct HostRecord { int type; std::vector<uint64_t> grid; std::vector<int32_t> map; std::vector<uint16_t> neigh; };

struct HostSearch {   // a codebook in the device layout (common.cuh SearchTab), host copy
    int type = 0, gd = 8, ngrid = 0;
    std::vector<int32_t> code3;
    std::vector<uint32_t> neigh;
    std::vector<uint16_t> glev;
};

std::vector<HostRecord> g_records;
std::vector<HostSearch> g_search;

// reads a gpuq_tables.bin (gpuq_tables.c:5-8 format); 0 ok, 2 open, 3 short read, 5 empty
int read_tables(const char * path, std::vector<HostRecord> & recs) {
    FILE * f = path ? std::fopen(path, "rb") : nullptr;
    if (!f) { set_err("gpuq_init: cannot open tables file '%s'", path ? path : "(null)"); return 2; }
    int32_t hdr[4];
    while (std::fread(hdr, sizeof(hdr), 1, f) == 1) {
        if (hdr[1] < 0 || hdr[2] < 0 || hdr[3] < 0 || hdr[1] > (1 << 20) || hdr[2] > (1 << 20) || hdr[3] > (1 << 24)) {
            std::fclose(f); set_err("gpuq_init: corrupt record header in '%s'", path); return 3;
        }
        HostRecord r{hdr[0], std::vector<uint64_t>(hdr[1]), std::vector<int32_t>(hdr[2]), std::vector<uint16_t>(hdr[3])};
        if (std::fread(r.grid.data(), 8, hdr[1], f) != (size_t) hdr[1] || std::fread(r.map.data(), 4, hdr[2], f) != (size_t) hdr[2] ||
            std::fread(r.neigh.data(), 2, hdr[3], f) != (size_t) hdr[3]) {
            std::fclose(f); set_err("gpuq_init: short read in '%s'", path); return 3;
        }
        recs.push_back(std::move(r));
    }
    std::fclose(f);
    if (recs.empty()) { set_err("gpuq_init: no tables in '%s'", path); return 5; }
    return 0;
}

// file record (ggml's kgrid / kmap / kneighbours) -> the device layout over the reachable level codes only
bool convert_search(const HostRecord & r, HostSearch & h) {
    const int gd = r.map.size() == 43692 ? 8 : r.map.size() == 4096 ? 4 : 0;
    if (!gd) { set_err("gpuq_init: type %d: unexpected map size %zu", r.type, r.map.size()); return false; }
    const int bits = gd == 8 ? 2 : 3, nlev = gd == 8 ? 3 : 8;
    h.type = r.type; h.gd = gd; h.ngrid = (int) r.grid.size();
    auto pack = [&](uint64_t p, bool * ok) {
        uint32_t lev = 0;
        for (int i = 0; i < gd; ++i) {
            const int v = (int) ((p >> (8 * i)) & 255);
            const int l = (v - 1) / 2;
            if (v < 1 || v % 2 == 0 || l >= nlev) *ok = false;
            lev |= (uint32_t) (l < 0 ? 0 : l) << (bits * i);
        }
        return lev;
    };
    bool ok = true;
    h.glev.resize(h.ngrid);
    for (int g = 0; g < h.ngrid; ++g) h.glev[g] = (uint16_t) pack(r.grid[g], &ok);
    if (!ok) { set_err("gpuq_init: type %d: grid point outside the 2l+1 lattice", r.type); return false; }
    int ncode = 1;
    for (int i = 0; i < gd; ++i) ncode *= nlev;
    h.code3.assign(ncode, 0);
    h.neigh.clear();
    for (int c = 0; c < ncode; ++c) {
        int u = 0, cc = c;
        for (int i = 0; i < gd; ++i) { u |= (cc % nlev) << (bits * i); cc /= nlev; }
        const int m = r.map[u];
        if (m >= 0) {
            if (m >= h.ngrid) { set_err("gpuq_init: type %d: map entry out of range", r.type); return false; }
            h.code3[c] = m;
            continue;
        }
        const size_t off = (size_t) (-m - 1);
        if (off >= r.neigh.size() || off + 1 + r.neigh[off] > r.neigh.size() || r.neigh[off] == 0) {
            set_err("gpuq_init: type %d: neighbour list out of range", r.type); return false;
        }
        const int n = r.neigh[off];
        if (n >= (1 << LIST_CNT_BITS) || h.neigh.size() >= ((size_t) 1 << (30 - LIST_CNT_BITS))) {
            set_err("gpuq_init: type %d: neighbour list too long for the device layout", r.type); return false;
        }
        h.code3[c] = -(int32_t) (((h.neigh.size() << LIST_CNT_BITS) | (size_t) n) + 1);
        h.neigh.push_back((uint32_t) n);
        for (int j = 1; j <= n; ++j) {
            const int gi = r.neigh[off + j];
            if (gi >= h.ngrid) { set_err("gpuq_init: type %d: neighbour index out of range", r.type); return false; }
            h.neigh.push_back(((uint32_t) gi << 16) | h.glev[gi]);
        }
    }
    h.neigh.push_back(0);   // pad word: the searches load the entry after a list's last one ahead of time
    return true;
}

// ------------------------------------------------------------------------------------------------ device state
constexpr int NSLOT = 2;

struct Device {
    int id = -1;
    bool ready = false;
    std::mutex mu;                         // the host API of one device runs one call at a time
    // tables
    struct DevSearch { int type; SearchTab tab; int32_t * code3; uint32_t * neigh; uint16_t * glev; };
    std::vector<DevSearch> search;
    struct DevGrid { int type; uint64_t * grid; };
    std::vector<DevGrid> dgrid;
    unsigned * status = nullptr;
    // pipeline
    cudaStream_t s_h2d = nullptr, s_run = nullptr, s_d2h = nullptr;
    cudaEvent_t ev_h2d[NSLOT] = {}, ev_run[NSLOT] = {}, ev_d2h[NSLOT] = {};
    void * d_src[NSLOT] = {}; size_t cap_src[NSLOT] = {};
    void * d_out[NSLOT] = {}; size_t cap_out[NSLOT] = {};
    void * h_out[NSLOT] = {}; size_t cap_hout[NSLOT] = {};   // pinned staging for pageable destinations
    void * h_src[NSLOT] = {}; size_t cap_hsrc[NSLOT] = {};   // pinned staging for pageable sources
    float * d_qw = nullptr; size_t cap_qw = 0;
    void * d_f32[NSLOT] = {}; size_t cap_f32[NSLOT] = {};   // staged sources: the chunk decoded to float32
    float * d_scale = nullptr; size_t cap_scale = 0;         // per-matrix second scales

    const SearchTab * tab(int type) const {
        const int want = type == IQ1_M ? IQ1_S : type;
        for (auto & s : search) if (s.type == want) return &s.tab;
        return nullptr;
    }
    const uint64_t * dq_grid(int type) const {
        const int want = 1000 + (type == IQ1_M ? IQ1_S : type);
        for (auto & g : dgrid) if (g.type == want) return g.grid;
        return nullptr;
    }
};

std::mutex g_mu;                                    // guards the device list
std::vector<std::unique_ptr<Device>> g_dev;         // every initialized device
std::vector<Device *> g_active;                     // the devices the host API fans out over (first = primary)

Device * find_dev(int id) {
    for (auto & d : g_dev) if (d->id == id) return d.get();
    return nullptr;
}

bool grow(void ** p, size_t * cap, size_t need, bool pinned = false) {
    if (need <= *cap) return true;
    if (*p) { if (pinned) cudaFreeHost(*p); else cudaFree(*p); }
    *p = nullptr; *cap = 0;
    const size_t sz = need + need / 8;   // headroom against one-byte regrowth
    const cudaError_t e = pinned ? cudaMallocHost(p, sz) : cudaMalloc(p, sz);
    if (e != cudaSuccess) { *p = nullptr; set_err("allocation of %zu bytes failed: %s", sz, cudaGetErrorString(e)); return false; }
    *cap = sz;
    return true;
}

int upload_tables(Device & d) {
    for (auto & r : g_records) {
        if (r.type >= 1000) {
            uint64_t * g = nullptr;
            if (cudaMalloc(&g, r.grid.size() * 8) != cudaSuccess) return 4;
            cudaMemcpy(g, r.grid.data(), r.grid.size() * 8, cudaMemcpyHostToDevice);
            d.dgrid.push_back({r.type, g});
        }
    }
    for (auto & h : g_search) {
        Device::DevSearch s{h.type, {}, nullptr, nullptr, nullptr};
        if (cudaMalloc(&s.code3, h.code3.size() * 4) != cudaSuccess || cudaMalloc(&s.neigh, h.neigh.size() * 4) != cudaSuccess ||
            cudaMalloc(&s.glev, h.glev.size() * 2) != cudaSuccess) return 4;
        cudaMemcpy(s.code3, h.code3.data(), h.code3.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(s.neigh, h.neigh.data(), h.neigh.size() * 4, cudaMemcpyHostToDevice);   // (includes the pad word)
        cudaMemcpy(s.glev, h.glev.data(), h.glev.size() * 2, cudaMemcpyHostToDevice);
        s.tab = SearchTab{s.code3, s.neigh, s.glev, h.ngrid};
        d.search.push_back(s);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

int init_device(int id) {
    Device * d = find_dev(id);
    if (d && d->ready) return 0;
    if (cudaSetDevice(id) != cudaSuccess) { set_err("gpuq_init: cudaSetDevice(%d) failed", id); return 1; }
    if (!d) { g_dev.emplace_back(new Device()); d = g_dev.back().get(); d->id = id; }
    if (std::getenv("GPUQ_FAIL_ALLOC")) { set_err("gpuq_init: allocation failure forced by GPUQ_FAIL_ALLOC"); return 4; }
    if (upload_tables(*d)) { set_err("gpuq_init: device %d: table upload failed", id); return 4; }
    if (cudaMalloc(&d->status, sizeof(unsigned)) != cudaSuccess) return 4;
    cudaMemset(d->status, 0, sizeof(unsigned));
    if (cudaStreamCreateWithFlags(&d->s_h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d->s_run, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d->s_d2h, cudaStreamNonBlocking) != cudaSuccess) return 4;
    for (int i = 0; i < NSLOT; ++i)
        if (cudaEventCreateWithFlags(&d->ev_h2d[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&d->ev_run[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&d->ev_d2h[i], cudaEventDisableTiming) != cudaSuccess) return 4;
    noalloc_prepare(id);   // gpuq_requantize_noalloc's scratch array: loaded here, at set-up
    d->ready = true;
    return 0;
}

// the current device's state (device API), or null
Device * current_device() {
    int id = -1;
    if (cudaGetDevice(&id) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    Device * d = find_dev(id);
    return d && d->ready ? d : nullptr;
}

size_t raw_bytes(int src, int64_t n) {
    if (elementwise_src(src) && n >= 0) return (size_t) n * (src == SRC_F32 ? 4 : 2);   // (exact for any count)
    const int bl = src_block_len(src);
    return bl && n >= 0 ? (size_t) (n / bl) * src_block_bytes(src) : 0;
}

bool type_ok(int type, int64_t n_per_row, const void * imatrix) {
    const int bb = block_bytes(type);
    if (!bb) { set_err("type %d is not quantized by this library", type); return false; }
    if (needs_search_tab(type)) {
        if (g_active.empty() || !g_active[0]->tab(type)) { set_err("type %d: no search tables (gpuq_init first)", type); return false; }
    }
    if (!imatrix && !takes_no_imatrix(type)) { set_err("type %d needs an importance matrix", type); return false; }
    if (n_per_row <= 0 || n_per_row % block_len(type)) { set_err("row length %lld is not a multiple of %d", (long long) n_per_row, block_len(type)); return false; }
    return true;
}

bool is_pinned(const void * p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) { cudaGetLastError(); return false; }
    return a.type == cudaMemoryTypeHost;
}

// one piece of a host call: matrices [m0, m1) whole, or rows [r0, r1) of matrix m0
struct Chunk { int64_t m0, m1, r0, r1; };

struct HostJob {
    int type, src;
    const uint8_t * raw;           // host source bytes
    uint8_t * dst;                 // host output bytes
    int64_t nmat, nrow, n_per_row;
    const float * imatrix;         // host, nmat x n_per_row, or null
    const float * mat_scale;       // host, nmat per-matrix scales applied after decoding, or null
    std::vector<Chunk> chunks;
    std::atomic<bool> cancel{false};   // set by a device worker that failed: the others stop before their next chunk
};

// host memcpy split over up to 8 threads for large pieces (one thread copies ~10 GB/s, less than a PCIe 5 link): the
// pageable sources into the pinned slots and the results out to pageable destinations
void host_copy(void * dst, const void * src, size_t n) {
    constexpr size_t PIECE = (size_t) 4 << 20;
    const int nt = (int) std::min<size_t>(8, n / PIECE);
    if (nt <= 1) { std::memcpy(dst, src, n); return; }
    std::vector<std::thread> th;
    const size_t per = (n / nt + 63) & ~(size_t) 63;
    for (int k = 1; k < nt; ++k) {
        const size_t a = per * k, b = std::min(n, a + per);
        if (a < b) th.emplace_back([=] { std::memcpy((uint8_t *) dst + a, (const uint8_t *) src + a, b - a); });
    }
    std::memcpy(dst, src, std::min(n, per));
    for (auto & t : th) t.join();
}

// chunks of about target_values each; the first is a quarter of that (a matrix or a quarter of the rows), so the
// pipeline's first copy - the one nothing overlaps - is short
std::vector<Chunk> make_chunks(int64_t nmat, int64_t nrow, int64_t n_per_row, int64_t target_values) {
    std::vector<Chunk> c;
    const int64_t per_mat = nrow * n_per_row;
    if (per_mat >= target_values) {
        const int64_t rows = std::max<int64_t>(1, target_values / n_per_row);
        const int64_t first = std::max<int64_t>(1, rows / 4);
        for (int64_t m = 0; m < nmat; ++m) {
            int64_t r = 0;
            if (m == 0 && first < rows && first < nrow) { c.push_back({0, 1, 0, first}); r = first; }
            for (; r < nrow; r += rows) c.push_back({m, m + 1, r, std::min(nrow, r + rows)});
        }
    } else {
        const int64_t mats = std::max<int64_t>(1, target_values / per_mat);
        const int64_t first = std::max<int64_t>(1, mats / 4);
        int64_t m = 0;
        if (first < mats && first < nmat) { c.push_back({0, first, 0, nrow}); m = first; }
        for (; m < nmat; m += mats) c.push_back({m, std::min(nmat, m + mats), 0, nrow});
    }
    return c;
}

int64_t chunk_values() {
    const char * e = std::getenv("GPUQ_CHUNK_MW");   // millions of weights a chunk
    const int64_t mw = e ? std::max<int64_t>(1, std::atoll(e)) : 64;
    return mw * 1000000;
}

// runs the chunks [c0, c1) of a job on one device through the 3-stream pipeline; false on error. Pinned caller
// buffers are copied directly; a pageable source chunk is first copied on the host into the slot's pinned staging
// buffer (while the other slot's kernel runs), a pageable destination is filled from the slot's pinned staging
// buffer once its device-to-host copy is done - so the copies overlap the kernels for numpy callers too.
bool run_chunks(Device & d, HostJob & j, size_t c0, size_t c1) {
    std::lock_guard<std::mutex> lk(d.mu);
    if (const char * f = std::getenv("GPUQ_FAIL_DEVICE")) {   // host-side fault injection: this device's worker fails
        if (std::atoi(f) == d.id) { set_err("device worker failure injected by GPUQ_FAIL_DEVICE"); return false; }
    }
    if (cudaSetDevice(d.id) != cudaSuccess) { set_err("cudaSetDevice(%d) failed", d.id); return false; }
    const int bs = block_len(j.type), bb = block_bytes(j.type);
    const int64_t nb_row = j.n_per_row / bs;
    const bool want_qw = j.imatrix && j.type != Q8_0 && j.type != F16;   // (both ignore it, as ggml_quantize_chunk)
    if (want_qw) {
        const size_t qb = (size_t) j.nmat * j.n_per_row * 4;
        if (!grow((void **) &d.d_qw, &d.cap_qw, qb)) return false;
        if (cudaMemcpyAsync(d.d_qw, j.imatrix, qb, cudaMemcpyHostToDevice, d.s_h2d) != cudaSuccess) { set_err("imatrix copy failed"); return false; }
    }
    // staged sources (and any source with per-matrix scales) are decoded to float32 by their own pass first
    const bool staged = !src_bytes32(j.src) || j.mat_scale;
    if (j.mat_scale) {
        if (!grow((void **) &d.d_scale, &d.cap_scale, (size_t) j.nmat * 4)) return false;
        if (cudaMemcpyAsync(d.d_scale, j.mat_scale, (size_t) j.nmat * 4, cudaMemcpyHostToDevice, d.s_h2d) != cudaSuccess) {
            set_err("scale copy failed"); return false;
        }
    }
    const DequantTab src_tab{d.dq_grid(j.src)};
    const bool src_pinned = is_pinned(j.raw), dst_pinned = is_pinned(j.dst);
    cudaMemsetAsync(d.status, 0, sizeof(unsigned), d.s_run);
    struct Pending { bool on = false; uint8_t * dst = nullptr; size_t bytes = 0; };
    Pending pend[NSLOT];
    bool ok = true;
    auto finish = [&](int slot) {   // host side of a slot's D2H: copy staged bytes to the caller's buffer
        if (!pend[slot].on) return;
        if (cudaEventSynchronize(d.ev_d2h[slot]) != cudaSuccess) ok = false;
        else if (!dst_pinned) host_copy(pend[slot].dst, d.h_out[slot], pend[slot].bytes);
        pend[slot].on = false;
    };
    // the imatrix and scale copies must land before the first kernel
    cudaEvent_t ev_qw = nullptr;
    cudaEventCreateWithFlags(&ev_qw, cudaEventDisableTiming);
    cudaEventRecord(ev_qw, d.s_h2d);
    cudaStreamWaitEvent(d.s_run, ev_qw, 0);
    for (size_t ci = c0; ci < c1 && ok; ++ci) {
        if (j.cancel.load(std::memory_order_relaxed)) { set_err("cancelled: another device of this call failed"); ok = false; break; }
        const Chunk & c = j.chunks[ci];
        const int slot = (int) ((ci - c0) % NSLOT);
        const int64_t rows = c.r1 - c.r0, mats = c.m1 - c.m0;
        const int64_t v0 = (c.m0 * j.nrow + c.r0) * j.n_per_row;
        const int64_t nv = mats * rows * j.n_per_row;
        const int64_t nblocks = nv / bs;
        const size_t in_bytes = raw_bytes(j.src, nv), out_bytes = (size_t) nblocks * bb;
        finish(slot);   // the slot's previous chunk: its bytes are out, its buffers free
        if (!grow(&d.d_src[slot], &d.cap_src[slot], in_bytes) || !grow(&d.d_out[slot], &d.cap_out[slot], out_bytes) ||
            (!dst_pinned && !grow(&d.h_out[slot], &d.cap_hout[slot], out_bytes, true)) ||
            (!src_pinned && !grow(&d.h_src[slot], &d.cap_hsrc[slot], in_bytes, true)) ||
            (staged && !grow(&d.d_f32[slot], &d.cap_f32[slot], (size_t) nv * 4))) { ok = false; break; }
        const uint8_t * hsrc = j.raw + raw_bytes(j.src, v0);
        if (!src_pinned) {   // (the slot's previous H2D is done: finish() waited for its D2H, which followed it)
            host_copy(d.h_src[slot], hsrc, in_bytes);
            hsrc = (const uint8_t *) d.h_src[slot];
        }
        // H2D once the kernel that last read this slot's source buffer is done
        cudaStreamWaitEvent(d.s_h2d, d.ev_run[slot], 0);
        if (cudaMemcpyAsync(d.d_src[slot], hsrc, in_bytes, cudaMemcpyHostToDevice, d.s_h2d) != cudaSuccess) {
            set_err("host-to-device copy failed"); ok = false; break;
        }
        cudaEventRecord(d.ev_h2d[slot], d.s_h2d);
        cudaStreamWaitEvent(d.s_run, d.ev_h2d[slot], 0);
        cudaStreamWaitEvent(d.s_run, d.ev_d2h[slot], 0);   // the output buffer's previous D2H is done
        if (staged && launch_stage(j.src, d.d_src[slot], (float *) d.d_f32[slot], nv, src_tab, j.mat_scale ? d.d_scale : nullptr,
                                   j.nrow * j.n_per_row, v0, d.s_run) != cudaSuccess) {
            set_err("source decode launch failed: %s", cudaGetErrorString(cudaGetLastError())); ok = false; break;
        }
        LaunchArgs a{};
        a.src_type = staged ? (int) SRC_F32 : j.src;
        a.src = staged ? d.d_f32[slot] : d.d_src[slot];
        a.qw = want_qw ? d.d_qw + c.m0 * j.n_per_row : nullptr;
        a.qw_mod = nb_row; a.qw_div = 1; a.qw_mat = rows * nb_row;
        a.out = d.d_out[slot];
        a.nblocks = nblocks;
        const SearchTab * t = d.tab(j.type);
        a.tab = t ? *t : SearchTab{};
        a.status = d.status;
        a.stream = d.s_run;
        a.n_per_row = j.n_per_row;
        if (launch_quantize(j.type, a) != cudaSuccess) { set_err("kernel launch failed: %s", cudaGetErrorString(cudaGetLastError())); ok = false; break; }
        cudaEventRecord(d.ev_run[slot], d.s_run);
        cudaStreamWaitEvent(d.s_d2h, d.ev_run[slot], 0);
        uint8_t * hdst = j.dst + (size_t) (v0 / bs) * bb;
        if (cudaMemcpyAsync(dst_pinned ? (void *) hdst : d.h_out[slot], d.d_out[slot], out_bytes, cudaMemcpyDeviceToHost, d.s_d2h) != cudaSuccess) {
            set_err("device-to-host copy failed"); ok = false; break;
        }
        cudaEventRecord(d.ev_d2h[slot], d.s_d2h);
        pend[slot] = {true, hdst, out_bytes};
    }
    for (int s = 0; s < NSLOT; ++s) finish(s);
    const cudaError_t e1 = cudaStreamSynchronize(d.s_run), e2 = cudaStreamSynchronize(d.s_d2h), e3 = cudaStreamSynchronize(d.s_h2d);
    cudaEventDestroy(ev_qw);
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess) { set_err("CUDA error: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e3)); return false; }
    if (!ok) return false;
    unsigned st = 0;
    cudaMemcpy(&st, d.status, sizeof(st), cudaMemcpyDeviceToHost);
    if (st) { set_err("device status 0x%x (no finite neighbour / off-grid code: non-finite input?)", st); return false; }
    return true;
}

size_t run_host_job(HostJob & j) {
    std::vector<Device *> devs;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        devs = g_active;
    }
    if (devs.empty()) { set_err("gpuq_init has not been called"); return 0; }
    const int bs = block_len(j.type);
    const size_t total = (size_t) j.nmat * j.nrow * (j.n_per_row / bs) * block_bytes(j.type);
    int cur = 0;
    cudaGetDevice(&cur);
    // shards: contiguous chunk ranges, one a device (experts / row ranges split evenly; no collective)
    const int64_t target = chunk_values();
    const int nd = (int) devs.size();
    j.chunks = make_chunks(j.nmat, j.nrow, j.n_per_row, nd > 1 ? std::min<int64_t>(target, std::max<int64_t>(bs, j.nmat * j.nrow * j.n_per_row / (2 * nd))) : target);
    const size_t nc = j.chunks.size();
    bool ok = true;
    if (nd == 1 || nc == 1) {
        ok = run_chunks(*devs[0], j, 0, nc);
    } else {
        std::vector<std::thread> th;
        std::vector<char> res(nd, 1);
        std::vector<std::string> errs(nd);
        for (int k = 0; k < nd; ++k) {
            const size_t a = nc * k / nd, b = nc * (k + 1) / nd;
            if (a >= b) continue;
            th.emplace_back([&, k, a, b] {
                res[k] = run_chunks(*devs[k], j, a, b);
                if (!res[k]) { errs[k] = t_err; j.cancel.store(true, std::memory_order_relaxed); }
            });
        }
        for (auto & t : th) t.join();
        // the first failure that was not a cancellation names the cause
        for (int k = nd - 1; k >= 0; --k)
            if (!res[k] && (ok || errs[k].rfind("cancelled", 0) != 0)) { ok = false; t_err = "device " + std::to_string(devs[k]->id) + ": " + errs[k]; }
    }
    cudaSetDevice(cur);
    return ok ? total : 0;
}

}  // namespace

const SearchTab * current_search_tab(int type, bool * device_ready) {
    Device * d = current_device();
    if (device_ready) *device_ready = d != nullptr;
    return d ? d->tab(type) : nullptr;
}

void set_last_error(const char * msg) { t_err = msg; }

}  // namespace gq

using namespace gq;

extern "C" {

int gpuq_init(const char * tables, int device) {
    std::lock_guard<std::mutex> lk(g_mu);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        set_err("gpuq_init: no CUDA device %d", device);
        return 1;
    }
    if (g_records.empty()) {
        std::vector<HostRecord> recs;
        const int rc = read_tables(tables, recs);
        if (rc) return rc;
        std::vector<HostSearch> srch;
        for (auto & r : recs) {
            if (r.type >= 1000) continue;
            HostSearch h;
            if (!convert_search(r, h)) return 3;
            srch.push_back(std::move(h));
        }
        g_records = std::move(recs);
        g_search = std::move(srch);
    }
    const int rc = init_device(device);
    if (rc) return rc;
    Device * d = find_dev(device);
    g_active.clear();
    g_active.push_back(d);
    cudaSetDevice(device);
    return 0;
}

int gpuq_init_devices(const char * tables, const int * devices, int ndev) {
    if (!devices || ndev <= 0) { set_err("gpuq_init_devices: empty device list"); return 1; }
    const int rc = gpuq_init(tables, devices[0]);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    std::vector<Device *> act{find_dev(devices[0])};
    for (int i = 1; i < ndev; ++i) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || devices[i] < 0 || devices[i] >= n) { set_err("gpuq_init_devices: no device %d", devices[i]); return 1; }
        const int r = init_device(devices[i]);
        if (r) return r;
        act.push_back(find_dev(devices[i]));
    }
    g_active = act;
    cudaSetDevice(devices[0]);
    return 0;
}

int gpuq_device_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return (int) g_active.size();
}

const char * gpuq_last_error(void) { return t_err.c_str(); }

unsigned gpuq_status(int reset) {
    Device * d = current_device();
    if (!d) return 0;
    unsigned st = 0;
    cudaMemcpy(&st, d->status, sizeof(st), cudaMemcpyDeviceToHost);
    if (reset) cudaMemset(d->status, 0, sizeof(unsigned));
    return st;
}

size_t gpuq_block_bytes(int type) { return (size_t) block_bytes(type); }

int gpuq_can_quantize(int type, int with_imatrix) {
    std::lock_guard<std::mutex> lk(g_mu);
    return type_ok(type, block_len(type), with_imatrix ? (const void *) 1 : nullptr) ? 1 : 0;
}

size_t gpuq_quantize_batch(int type, const float * src, void * dst, int64_t nmat, int64_t nrow, int64_t n_per_row,
                           const float * imatrix) {
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (nmat <= 0 || nrow <= 0 || !src || !dst || !type_ok(type, n_per_row, imatrix)) {
            if (nmat <= 0 || nrow <= 0) set_err("empty batch");
            return 0;
        }
    }
    HostJob j{type, SRC_F32, (const uint8_t *) src, (uint8_t *) dst, nmat, nrow, n_per_row, imatrix, nullptr, {}};
    return run_host_job(j);
}

size_t gpuq_quantize(int type, const float * src, void * dst, int64_t nrow, int64_t n_per_row, const float * imatrix) {
    return gpuq_quantize_batch(type, src, dst, 1, nrow, n_per_row, imatrix);
}

int gpuq_can_dequantize(int src) { return src_block_len(src) > 0 ? 1 : 0; }

}  // extern "C"

namespace {
// checks of a requantize call from host bytes (the callers hold no lock)
bool requantize_args_ok(int src, const void * raw, int type, const void * dst, int64_t nmat, int64_t nrow,
                        int64_t n_per_row, const float * imatrix) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int sl = src_block_len(src);
    if (!sl) { set_err("source type %d cannot be read on the GPU", src); return false; }
    if (g_active.empty()) { set_err("gpuq_init has not been called"); return false; }
    if (nmat <= 0 || nrow <= 0) { set_err("empty batch"); return false; }
    if (!raw || !dst) { set_err("null source or destination"); return false; }
    if (!type_ok(type, n_per_row, imatrix)) return false;
    // (an F16 target takes rows of any length from a source without blocks: F16 is the fallback for such rows)
    if (n_per_row % sl && !(type == F16 && elementwise_src(src))) {
        set_err("row length %lld is not a multiple of source type %d's %d-value blocks", (long long) n_per_row, src, sl);
        return false;
    }
    if (is_block_src(src) && src != IQ4_XS && !is_kquant(src) && !g_active[0]->dq_grid(src)) {
        set_err("source type %d: no dequant grid (gpuq_init first)", src); return false;
    }
    return true;
}
}  // namespace

extern "C" {

size_t gpuq_requantize_batch(int src, const void * raw, int type, void * dst, int64_t nmat, int64_t nrow,
                             int64_t n_per_row, const float * imatrix) {
    if (!requantize_args_ok(src, raw, type, dst, nmat, nrow, n_per_row, imatrix)) return 0;
    HostJob j{type, src, (const uint8_t *) raw, (uint8_t *) dst, nmat, nrow, n_per_row, imatrix, nullptr, {}};
    return run_host_job(j);
}

size_t gpuq_requantize_scaled_batch(int src, const void * raw, int type, void * dst, int64_t nmat, int64_t nrow,
                                    int64_t n_per_row, const float * imatrix, const float * mat_scale) {
    if (!requantize_args_ok(src, raw, type, dst, nmat, nrow, n_per_row, imatrix)) return 0;
    if (!mat_scale) { set_err("gpuq_requantize_scaled_batch: null scales"); return 0; }
    HostJob j{type, src, (const uint8_t *) raw, (uint8_t *) dst, nmat, nrow, n_per_row, imatrix, mat_scale, {}};
    return run_host_job(j);
}

size_t gpuq_requantize(int src, const void * raw, int type, void * dst, int64_t nrow, int64_t n_per_row,
                       const float * imatrix) {
    return gpuq_requantize_batch(src, raw, type, dst, 1, nrow, n_per_row, imatrix);
}

size_t gpuq_quantize_dev(int type, const float * d_x, void * d_dst, int64_t nblocks, const float * d_qw, int64_t qw_mod,
                         int64_t qw_div, void * stream) {
    // the reference's device API takes the 256-block i-quants; this library also takes the k-quants (Q2_K..Q6_K, which
    // its gpuq_can_dequantize_type reports, so LDLQ callers run them on the GPU); not the 32-block IQ4_NL and Q8_0
    if (!block_bytes(type) || block_len(type) != QK || nblocks <= 0 || qw_mod <= 0 || qw_div <= 0 || !d_x || !d_dst) {
        set_err("gpuq_quantize_dev: unsupported type %d or bad arguments", type);
        return 0;
    }
    Device * d = current_device();
    if (!d) { set_err("gpuq_quantize_dev: current device not initialized"); return 0; }
    if (needs_search_tab(type) && !d->tab(type)) { set_err("gpuq_quantize_dev: no tables for type %d", type); return 0; }
    if (!d_qw && !takes_no_imatrix(type)) { set_err("gpuq_quantize_dev: type %d needs importance weights", type); return 0; }
    LaunchArgs a{};
    a.src_type = SRC_F32; a.src = d_x; a.qw = d_qw; a.qw_mod = qw_mod; a.qw_div = qw_div; a.qw_mat = INT64_MAX;
    a.out = d_dst; a.nblocks = nblocks;
    const SearchTab * t = d->tab(type);
    a.tab = t ? *t : SearchTab{};
    a.status = d->status; a.stream = (cudaStream_t) stream;
    if (launch_quantize(type, a) != cudaSuccess) { set_err("gpuq_quantize_dev: launch failed"); return 0; }
    return (size_t) nblocks * block_bytes(type);
}

size_t gpuq_requantize_dev(int src, const void * d_raw, int type, void * d_dst, int64_t nmat, int64_t nrow,
                           int64_t n_per_row, const float * d_imatrix, void * stream) {
    const int64_t n = nmat * nrow * n_per_row;
    if (nmat <= 0 || nrow <= 0 || !d_raw || !d_dst || (n % 32 && !(type == F16 && elementwise_src(src)))) {
        set_err("gpuq_requantize_dev: bad arguments");
        return 0;
    }
    if (!src_bytes32(src)) {   // (a staged source needs a float32 buffer: the device API keeps no scratch)
        set_err("gpuq_requantize_dev: source type %d is decoded by its own pass: gpuq_dequantize_src_dev into a float32 "
                "buffer, then gpuq_requantize_dev with source 0 (F32)", src);
        return 0;
    }
    Device * d = current_device();
    if (!d) { set_err("gpuq_requantize_dev: current device not initialized"); return 0; }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!type_ok(type, n_per_row, d_imatrix)) return 0;
    }
    const int64_t nb_row = n_per_row / block_len(type);
    LaunchArgs a{};
    a.src_type = src; a.src = d_raw;
    a.qw = type == Q8_0 || type == F16 ? nullptr : d_imatrix;
    a.qw_mod = nb_row; a.qw_div = 1; a.qw_mat = nrow * nb_row;
    a.out = d_dst; a.nblocks = n / block_len(type); a.n_per_row = n_per_row;
    const SearchTab * t = d->tab(type);
    a.tab = t ? *t : SearchTab{};
    a.status = d->status; a.stream = (cudaStream_t) stream;
    if (launch_quantize(type, a) != cudaSuccess) { set_err("gpuq_requantize_dev: launch failed"); return 0; }
    return (size_t) a.nblocks * block_bytes(type);
}

int gpuq_can_dequantize_type(int type) {
    switch (type) {
        case IQ2_XXS: case IQ2_XS: case IQ2_S: case IQ3_XXS: case IQ3_S: case IQ1_S: case IQ1_M: {
            std::lock_guard<std::mutex> lk(g_mu);
            return !g_active.empty() && g_active[0]->dq_grid(type) ? 1 : 0;
        }
        case IQ4_XS: case Q2_K: case Q3_K: case Q4_K: case Q5_K: case Q6_K: return 1;
        default: return 0;
    }
}

size_t gpuq_dequantize_dev(int type, const void * d_q, float * d_out, int64_t nblocks, void * stream) {
    if (!gpuq_can_dequantize_type(type) || nblocks <= 0 || !d_q || !d_out) { set_err("gpuq_dequantize_dev: bad arguments"); return 0; }
    Device * d = current_device();
    if (!d) { set_err("gpuq_dequantize_dev: current device not initialized"); return 0; }
    if (launch_dequant(type, d_q, d_out, nblocks, DequantTab{d->dq_grid(type)}, (cudaStream_t) stream) != cudaSuccess) {
        set_err("gpuq_dequantize_dev: launch failed");
        return 0;
    }
    return (size_t) nblocks * QK * 4;
}

size_t gpuq_dequantize_error_dev(int type, const void * d_q, const float * d_blk, void * d_err, int f64, int64_t nblocks,
                                 void * stream) {
    if (!gpuq_can_dequantize_type(type) || nblocks <= 0 || !d_q || !d_blk || !d_err) {
        set_err("gpuq_dequantize_error_dev: bad arguments");
        return 0;
    }
    Device * d = current_device();
    if (!d) { set_err("gpuq_dequantize_error_dev: current device not initialized"); return 0; }
    if (launch_dequant_error(type, d_q, d_blk, d_err, f64 != 0, nblocks, DequantTab{d->dq_grid(type)}, (cudaStream_t) stream) != cudaSuccess) {
        set_err("gpuq_dequantize_error_dev: launch failed");
        return 0;
    }
    return (size_t) nblocks * QK * (f64 ? 8 : 4);
}

namespace {
bool misaligned(const void * p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }
}  // namespace

size_t gpuq_ldlq_scale_dev(const double * d_err, const double * d_rd, double * d_es, int64_t ngroups, int64_t rows,
                           int64_t nsteps, int64_t kdim, int64_t step, void * stream) {
    if (!d_err || !d_rd || !d_es || ngroups <= 0 || rows <= 0 || nsteps <= 0 || step < 0 || step >= nsteps ||
        (kdim != 256 && kdim != 32 && kdim != 8) || misaligned(d_err, 16) || misaligned(d_rd, 16) || misaligned(d_es, 16)) {
        set_err("gpuq_ldlq_scale_dev: bad arguments (kdim 256, 32 or 8; 0 <= step < nsteps; every pointer 16-byte aligned)");
        return 0;
    }
    const cudaError_t e = launch_ldlq_scale(d_err, d_rd, d_es, ngroups, rows, nsteps, (int) kdim, step, (cudaStream_t) stream);
    if (e != cudaSuccess) { set_err("gpuq_ldlq_scale_dev: launch failed: %s", cudaGetErrorString(e)); return 0; }
    return (size_t) ngroups * rows * kdim * 8;
}

size_t gpuq_ldlq_update_dev(const double * d_es, const double * d_u, float * d_w, int64_t ngroups, int64_t rows,
                            int64_t ne0, int64_t kdim, int64_t step, void * stream) {
    if (!d_es || !d_u || !d_w || ngroups <= 0 || rows <= 0 || ne0 <= 0 || ne0 % QK || (kdim != 256 && kdim != 32 && kdim != 8) ||
        step < 0 || (step + 1) * kdim >= ne0 || misaligned(d_es, 16) || misaligned(d_u, 16) || misaligned(d_w, 8)) {
        set_err("gpuq_ldlq_update_dev: bad arguments (kdim 256, 32 or 8; columns left after step; ne0 %% 256 == 0; Es "
                "and U 16-byte aligned, W 8-byte aligned)");
        return 0;
    }
    const cudaError_t e = launch_ldlq_update(d_es, d_u, d_w, ngroups, rows, ne0, (int) kdim, step, (cudaStream_t) stream);
    if (e != cudaSuccess) { set_err("gpuq_ldlq_update_dev: launch failed: %s", cudaGetErrorString(e)); return 0; }
    return (size_t) ngroups * rows * (ne0 - (step + 1) * kdim) * 4;
}

size_t gpuq_ldlq_sub_weff_dev(const float * d_blk, const float * d_qw, int64_t qw_div, float * d_weff, int64_t rows,
                              void * stream) {
    if (!d_blk || !d_qw || !d_weff || rows <= 0 || qw_div <= 0) { set_err("gpuq_ldlq_sub_weff_dev: bad arguments"); return 0; }
    const cudaError_t e = launch_sub_weff(d_blk, d_qw, qw_div, d_weff, rows, (cudaStream_t) stream);
    if (e != cudaSuccess) { set_err("gpuq_ldlq_sub_weff_dev: launch failed: %s", cudaGetErrorString(e)); return 0; }
    return (size_t) rows * QK * 4;
}

size_t gpuq_ldlq_sub_points_dev(const float * d_blk, const float * d_weff, void * d_q, double * d_err, int64_t rows, int sub,
                                int c0, int scale_search, void * stream) {
    if (!d_blk || !d_weff || !d_q || !d_err || rows <= 0 || (sub != 32 && sub != 8) || c0 < 0 || c0 % sub ||
        c0 + sub > QK || scale_search < 0 || scale_search > 15) {
        set_err("gpuq_ldlq_sub_points_dev: bad arguments (sub 32 or 8, c0 a multiple of sub below 256, scale_search 0..15)");
        return 0;
    }
    Device * d = current_device();
    const uint64_t * grid = d ? d->dq_grid(IQ2_XXS) : nullptr;
    if (!grid) { set_err("gpuq_ldlq_sub_points_dev: no IQ2_XXS grid (gpuq_init first)"); return 0; }
    const cudaError_t e = launch_sub_points(d_blk, d_weff, (uint8_t *) d_q, d_err, rows, sub, c0, scale_search, grid,
                                            (cudaStream_t) stream);
    if (e != cudaSuccess) { set_err("gpuq_ldlq_sub_points_dev: launch failed: %s", cudaGetErrorString(e)); return 0; }
    return (size_t) rows * sub * 8;
}

size_t gpuq_dgemm_batched_dev(int tri, int64_t M, int64_t N, int64_t K, double alpha, const double * d_a, int64_t lda,
                              const double * d_b, int64_t ldb, double beta, double * d_c, int64_t ldc, int64_t batch,
                              int64_t stride_a, int64_t stride_b, int64_t stride_c, void * stream) {
    if (tri < 0 || tri > 2 || M <= 0 || N <= 0 || K <= 0 || !d_a || !d_b || !d_c || (K & 1) || (N & 1) || (lda & 1) ||
        (ldb & 1) || lda < K || ldb < N || ldc < N || (tri == 1 && K != N) || (tri == 2 && K != M) ||
        batch <= 0 || batch > 65535 || (batch > 1 && ((stride_a & 1) || (stride_b & 1))) ||
        misaligned(d_a, 16) || misaligned(d_b, 16) || misaligned(d_c, 8)) {
        set_err("gpuq_dgemm_dev: bad arguments (tri 0, 1 (B lower, K == N) or 2 (A lower, K == M); K, N, lda, ldb even; "
                "A and B 16-byte aligned)");
        return 0;
    }
    const cudaError_t e = launch_dgemm(tri, d_a, lda, d_b, ldb, d_c, ldc, M, N, K, alpha, beta, batch, stride_a, stride_b,
                                       stride_c, (cudaStream_t) stream);
    if (e != cudaSuccess) { set_err("gpuq_dgemm_dev: launch failed: %s", cudaGetErrorString(e)); return 0; }
    return (size_t) batch * M * N * 8;
}

size_t gpuq_dgemm_dev(int tri, int64_t M, int64_t N, int64_t K, double alpha, const double * d_a, int64_t lda,
                      const double * d_b, int64_t ldb, double beta, double * d_c, int64_t ldc, void * stream) {
    return gpuq_dgemm_batched_dev(tri, M, N, K, alpha, d_a, lda, d_b, ldb, beta, d_c, ldc, 1, 0, 0, 0, stream);
}

size_t gpuq_xtx_scratch_bytes(int src, int64_t rows, int64_t dim, int scaled) {
    if ((src != SRC_F32 && src != SRC_BF16) || rows <= 0 || dim <= 0) return 0;
    return xtx_scratch_bytes(src, rows, dim, scaled != 0);
}

size_t gpuq_xtx_dev(int src, const void * d_x, int64_t ld_x, const float * d_scale, int64_t rows, int64_t dim, double * d_h,
                    int accumulate, void * d_scratch, size_t scratch_bytes, void * stream) {
    const size_t need = gpuq_xtx_scratch_bytes(src, rows, dim, d_scale != nullptr);
    const size_t esz = src == SRC_BF16 ? 2 : 4;
    if (!need || !d_x || !d_h || !d_scratch || ld_x < dim || scratch_bytes < need || misaligned(d_scratch, 16) ||
        misaligned(d_x, esz) || misaligned(d_h, 8) || misaligned(d_scale, 4)) {
        set_err("gpuq_xtx_dev: bad arguments (source 0 (F32) or 30 (BF16), ld_x >= dim, scratch of "
                "gpuq_xtx_scratch_bytes bytes, 16-byte aligned)");
        return 0;
    }
    Device * d = current_device();
    if (!d) { set_err("gpuq_xtx_dev: current device not initialized"); return 0; }
    const cudaError_t e = launch_xtx(src, d_x, ld_x, d_scale, rows, dim, d_h, accumulate != 0, d_scratch, scratch_bytes,
                                     d->status, (cudaStream_t) stream);
    if (e != cudaSuccess) { set_err("gpuq_xtx_dev: launch failed: %s", cudaGetErrorString(e)); return 0; }
    return (size_t) rows * dim * esz;
}

size_t gpuq_dequantize_src_dev(int src, const void * d_raw, float * d_out, int64_t n, void * stream) {
    const int sl = src_block_len(src);
    if (!sl || n <= 0 || n % sl || n % 32 || !d_raw || !d_out) { set_err("gpuq_dequantize_src_dev: bad arguments"); return 0; }
    DequantTab tab{nullptr};
    if (is_block_src(src)) {
        Device * d = current_device();
        tab.grid = d ? d->dq_grid(src) : nullptr;
        if (!tab.grid && !(src == IQ4_XS || is_kquant(src))) { set_err("gpuq_dequantize_src_dev: no dequant grid for source type %d (gpuq_init first)", src); return 0; }
    }
    if (launch_decode(src, d_raw, d_out, n, tab, (cudaStream_t) stream) != cudaSuccess) { set_err("gpuq_dequantize_src_dev: launch failed"); return 0; }
    return (size_t) n * 4;
}

}  // extern "C"
