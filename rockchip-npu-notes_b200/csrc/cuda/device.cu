// device.cu -- CUDA implementation of the host/device seam (b2_device.h).
//
// One b2_dev per opened handle: a device ordinal, a non-blocking stream (or a caller's stream),
// and a few status words in host-mapped pinned memory that kernels set with plain stores (so
// no system-scope atomics are needed and the host reads them after a stream sync without a copy).
// b2d_linear picks the kernel for the shape: the weight-streaming GEMV for M <= 8, the persistent
// tcgen05 GEMM otherwise, plus the separate epilogue kernel for the unfused (CO_SEPARATE) arm.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <new>

#include "../b2_device.h"
#include "aux_kernels.h"
#include "common.cuh"
#include "gemm_sm100.h"
#include "gemv.h"
#include "graph_kernels.h"
#include "plan_kernels.h"
#include "ksplit.h"
#include "rocket_b200.h"

struct b2_dev {
    int ordinal;
    int sm_count;
    cudaStream_t own;
    cudaStream_t stream;
    unsigned *flags;        // host pointer of the mapped status words
    unsigned *flags_dev;    // the same words as seen by kernels
    b2::gemv::Scratch gemv; // tile sums and block counters of long-K small-M launches
    __half *gate_table;     // SiLU / GELU gates of every FP16 input (common.cuh)
    // cube entries: tensor maps of the input views and the output tile table (first use allocates)
    void *cube_dev;         // device copy: [B2D_CUBE_MAX_VIEWS] CUtensorMap, then [..] CubeOut
    void *cube_host;        // pinned staging of the same bytes (= what the device copy holds)
    b2k_cube_tile *cube_key;   // [B2D_CUBE_MAX_VIEWS] the input view each device map describes
    unsigned cube_maps, cube_outs;   // slots the device copy holds valid contents for
    // side stream of banded input copies (first use creates it; none if creation failed)
    cudaStream_t side;
    cudaEvent_t fork, side_ev[B2D_SIDE_EVENTS];
    bool side_tried;
};

namespace {

inline bool set_device(const b2_dev *d) { return d && cudaSetDevice(d->ordinal) == cudaSuccess; }

inline int rc_of(cudaError_t e) {
    if (e == cudaSuccess) return 0;
    if (e == cudaErrorMemoryAllocation) return ROCKET_E_NOMEM;
    return ROCKET_E_DEVICE;
}

inline int flag_of_bit(uint32_t bit) {
    switch (bit) {
        case B2D_ST_TIMEOUT: return b2::FLAG_TIMEOUT;
        case B2D_ST_NONFINITE_OUTPUT: return b2::FLAG_NONFINITE_OUTPUT;
        case B2D_ST_NONFINITE_INPUT: return b2::FLAG_NONFINITE_INPUT;
        case B2D_ST_GUARD: return b2::FLAG_GUARD;
        case B2D_ST_SCAN_OUTPUT: return b2::FLAG_SCAN_OUTPUT;
        default: return -1;
    }
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int b2d_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int b2d_open(int ordinal, b2_dev **out) {
    *out = nullptr;
    if (ordinal < 0 || ordinal >= b2d_device_count()) return ROCKET_E_DEVICE;
    if (cudaSetDevice(ordinal) != cudaSuccess) return ROCKET_E_DEVICE;
    b2_dev *d = new (std::nothrow) b2_dev();
    if (!d) return ROCKET_E_NOMEM;
    d->ordinal = ordinal;
    if (cudaDeviceGetAttribute(&d->sm_count, cudaDevAttrMultiProcessorCount, ordinal) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d->own, cudaStreamNonBlocking) != cudaSuccess) {
        delete d;
        return ROCKET_E_DEVICE;
    }
    d->stream = d->own;
    if (cudaHostAlloc(reinterpret_cast<void **>(&d->flags), b2::FLAG_COUNT * sizeof(unsigned),
                      cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void **>(&d->flags_dev), d->flags, 0) != cudaSuccess) {
        if (d->flags) cudaFreeHost(d->flags);
        cudaStreamDestroy(d->own);
        delete d;
        return ROCKET_E_DEVICE;
    }
    memset(d->flags, 0, b2::FLAG_COUNT * sizeof(unsigned));
    // long-K small-M scratch: allocated once per handle (a launch recorded into a CUDA graph keeps
    // its address); the counters start at zero and every launch leaves them at zero
    void *ts = nullptr, *tc = nullptr;
    if (cudaMalloc(&ts, (size_t)b2::gemv::TSUM_FLOATS * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&tc, (size_t)b2::gemv::TCOUNT_WORDS * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(tc, 0, (size_t)b2::gemv::TCOUNT_WORDS * sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        if (ts) cudaFree(ts);
        if (tc) cudaFree(tc);
        cudaFreeHost(d->flags);
        cudaStreamDestroy(d->own);
        delete d;
        return ROCKET_E_NOMEM;
    }
    d->gemv.tsum = static_cast<float *>(ts);
    d->gemv.tcount = static_cast<unsigned *>(tc);
    void *gt = nullptr;
    if (cudaMalloc(&gt, (size_t)b2::GATE_TABLE_ENTRIES * sizeof(__half)) != cudaSuccess ||
        b2::graph::fill_gate_table(static_cast<__half *>(gt), d->stream) != cudaSuccess ||
        cudaStreamSynchronize(d->stream) != cudaSuccess) {
        cudaGetLastError();
        if (gt) cudaFree(gt);
        cudaFree(ts);
        cudaFree(tc);
        cudaFreeHost(d->flags);
        cudaStreamDestroy(d->own);
        delete d;
        return ROCKET_E_NOMEM;
    }
    d->gate_table = static_cast<__half *>(gt);
    if (b2::rkplan::prepare() != cudaSuccess) cudaGetLastError();   // plan tasks then report the launch error
    *out = d;
    return 0;
}

void b2d_close(b2_dev *d) {
    if (!d) return;
    set_device(d);
    cudaStreamSynchronize(d->stream);
    if (d->side) {
        cudaStreamSynchronize(d->side);
        cudaStreamDestroy(d->side);
        cudaEventDestroy(d->fork);
        for (unsigned i = 0; i < B2D_SIDE_EVENTS; ++i) cudaEventDestroy(d->side_ev[i]);
    }
    cudaStreamDestroy(d->own);
    cudaFreeHost(d->flags);
    cudaFree(d->gemv.tsum);
    cudaFree(d->gemv.tcount);
    cudaFree(d->gate_table);
    if (d->cube_dev) cudaFree(d->cube_dev);
    if (d->cube_host) cudaFreeHost(d->cube_host);
    free(d->cube_key);
    delete d;
}

int b2d_set_stream(b2_dev *d, void *stream) {
    if (!d) return ROCKET_E_SHAPE;
    d->stream = stream ? static_cast<cudaStream_t>(stream) : d->own;
    return 0;
}

void *b2d_stream(b2_dev *d) { return d ? static_cast<void *>(d->stream) : nullptr; }
int b2d_ordinal(b2_dev *d) { return d ? d->ordinal : -1; }
int b2d_sm_count(b2_dev *d) { return d ? d->sm_count : 0; }

int b2d_malloc(b2_dev *d, size_t bytes, void **out) {
    *out = nullptr;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return ROCKET_E_NOMEM;
    }
    if (cudaMemsetAsync(p, 0, bytes, d->stream) != cudaSuccess || cudaStreamSynchronize(d->stream) != cudaSuccess) {
        cudaFree(p);
        return ROCKET_E_DEVICE;
    }
    *out = p;
    return 0;
}

void b2d_free(b2_dev *d, void *ptr) {
    if (!ptr || !set_device(d)) return;
    cudaStreamSynchronize(d->stream);
    cudaFree(ptr);
}

void *b2d_host_alloc(size_t bytes) {
    void *p = nullptr;
    if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

void b2d_host_free(void *ptr) {
    if (ptr) cudaFreeHost(ptr);
}

int b2d_copy_2d(b2_dev *d, void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows,
                int kind) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!rows || !width) return 0;
    const cudaMemcpyKind k = kind == B2D_H2D ? cudaMemcpyHostToDevice
                             : kind == B2D_D2H ? cudaMemcpyDeviceToHost
                                               : cudaMemcpyDeviceToDevice;
    cudaError_t e;
    if (dpitch == width && spitch == width) e = cudaMemcpyAsync(dst, src, width * rows, k, d->stream);
    else e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, k, d->stream);
    return rc_of(e);
}

// The side stream and its events, created on first use; false (and no side stream) if any creation
// failed, in which case banded copies run on the handle's stream.
static bool side_ready(b2_dev *d) {
    if (d->side || d->side_tried) return d->side != nullptr;
    d->side_tried = true;
    cudaStream_t s = nullptr;
    cudaEvent_t ev[B2D_SIDE_EVENTS + 1] = {};
    bool ok = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess;
    unsigned made = 0;
    for (; ok && made <= B2D_SIDE_EVENTS; ++made)
        ok = cudaEventCreateWithFlags(&ev[made], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        for (unsigned i = 0; i < made; ++i)
            if (ev[i]) cudaEventDestroy(ev[i]);
        if (s) cudaStreamDestroy(s);
        return false;
    }
    d->side = s;
    d->fork = ev[B2D_SIDE_EVENTS];
    for (unsigned i = 0; i < B2D_SIDE_EVENTS; ++i) d->side_ev[i] = ev[i];
    return true;
}

int b2d_copy_side(b2_dev *d, void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows,
                  int kind, unsigned ev) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (ev >= B2D_SIDE_EVENTS) return ROCKET_E_SHAPE;
    if (!side_ready(d)) return b2d_copy_2d(d, dst, dpitch, src, spitch, width, rows, kind);
    const cudaMemcpyKind k = kind == B2D_H2D ? cudaMemcpyHostToDevice
                             : kind == B2D_D2H ? cudaMemcpyDeviceToHost
                                               : cudaMemcpyDeviceToDevice;
    cudaError_t e = cudaEventRecord(d->fork, d->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->side, d->fork, 0);
    if (e == cudaSuccess && rows && width)
        e = (dpitch == width && spitch == width) ? cudaMemcpyAsync(dst, src, width * rows, k, d->side)
                                                 : cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, k, d->side);
    if (e == cudaSuccess) e = cudaEventRecord(d->side_ev[ev], d->side);
    return rc_of(e);
}

int b2d_wait_side(b2_dev *d, unsigned ev) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (ev >= B2D_SIDE_EVENTS) return ROCKET_E_SHAPE;
    if (!d->side) return 0;   // the copies went to the handle's stream
    return rc_of(cudaStreamWaitEvent(d->stream, d->side_ev[ev], 0));
}

int b2d_memset(b2_dev *d, void *ptr, int value, size_t bytes) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    return rc_of(cudaMemsetAsync(ptr, value, bytes, d->stream));
}

int b2d_sync(b2_dev *d) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    return cudaStreamSynchronize(d->stream) == cudaSuccess ? 0 : ROCKET_E_DEVICE;
}

uint32_t b2d_status(b2_dev *d, int clear) {
    if (!d) return 0;
    volatile unsigned *f = d->flags;
    uint32_t bits = 0;
    if (f[b2::FLAG_TIMEOUT]) bits |= B2D_ST_TIMEOUT;
    if (f[b2::FLAG_NONFINITE_OUTPUT]) bits |= B2D_ST_NONFINITE_OUTPUT;
    if (f[b2::FLAG_NONFINITE_INPUT]) bits |= B2D_ST_NONFINITE_INPUT;
    if (f[b2::FLAG_GUARD]) bits |= B2D_ST_GUARD;
    if (f[b2::FLAG_SCAN_OUTPUT]) bits |= B2D_ST_SCAN_OUTPUT;
    if (clear) {
        for (int i = 0; i < b2::FLAG_COUNT; ++i) f[i] = 0;
        // A launch that timed out may have left long-K block counters raised: the next launch on
        // the stream must find them at zero.
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if ((bits & B2D_ST_TIMEOUT) && set_device(d) && cudaStreamIsCapturing(d->stream, &cs) == cudaSuccess &&
            cs == cudaStreamCaptureStatusNone)
            cudaMemsetAsync(d->gemv.tcount, 0, (size_t)b2::gemv::TCOUNT_WORDS * sizeof(unsigned), d->stream);
    }
    return bits;
}

void b2d_status_merge(b2_dev *d, uint32_t bits) {
    if (!d) return;
    volatile unsigned *f = d->flags;
    for (uint32_t b = 1; b <= B2D_ST_SCAN_OUTPUT; b <<= 1)
        if (bits & b) f[flag_of_bit(b)] = 1;
}

// ----------------------------------------------------------------------------- Linear dispatch
static bool use_gemv(const b2k_linear *a) { return a->m <= B2D_GEMV_MAX_M; }

int b2d_linear_config(b2_dev *d, const b2k_linear *a, b2k_config *cfg) {
    if (!d || !a || !cfg) return ROCKET_E_SHAPE;
    memset(cfg, 0, sizeof(*cfg));
    if (use_gemv(a)) {
        cfg->kernel = 1;
        cfg->tile_m = a->m;
        cfg->tile_n = 8;
        cfg->tile_k = 256;
        cfg->grid = b2::gemv::grid_for((int)a->m, (int)a->n, (int)a->k, (long long)a->ldw, d->sm_count);
        cfg->stages = b2::gemv::stream_stages((int)a->m, (int)a->n, (int)a->k, (long long)a->ldw);
    } else {
        cfg->kernel = 0;
        b2::gemm::config_for((int)a->m, (int)a->n, d->sm_count, &cfg->tile_m, &cfg->tile_n, &cfg->stages);
        cfg->tile_k = b2::gemm::TILE_K;
        cfg->grid = b2::gemm::grid_for((int)a->m, (int)a->n, d->sm_count);
    }
    return 0;
}

static bool linear_args_ok(const b2k_linear *a) {
    return a->m && a->n && a->k && a->x && a->w && a->ldx % 8 == 0 && a->ldw % 8 == 0 && a->ldx >= a->k &&
           a->ldw >= a->k && aligned16(a->x) && aligned16(a->w) && a->m <= (1u << 24) && a->n <= (1u << 24) &&
           a->k <= (1u << 24);
}

// One launch of the weight-streaming GEMV (M <= 8) or the GEMM in output mode `out_mode`, writing
// y/ldy (FP16 modes) or a->partial (OUT_RAW32). The bias is applied in OUT_FINAL only; the residual
// and gate fields go to the GEMM's epilogue only with `extra`.
static cudaError_t launch_core(b2_dev *d, const b2k_linear *a, int out_mode, bool fold, void *y, size_t ldy,
                               bool extra) {
    const __half *bias = static_cast<const __half *>(a->bias);
    if (use_gemv(a)) {
        b2::gemv::Params p = {};
        p.M = (int)a->m; p.N = (int)a->n; p.K = (int)a->k;
        p.x = static_cast<const __half *>(a->x); p.ldx = (long long)a->ldx;
        p.w = static_cast<const __half *>(a->w); p.ldw = (long long)a->ldw;
        p.bias = out_mode == b2::gemv::OUT_FINAL ? bias : nullptr;
        p.y = static_cast<__half *>(y); p.ldy = (long long)ldy;
        p.partial = a->partial; p.ldp = (long long)a->ldp;
        p.out_mode = out_mode; p.post = a->post; p.fold = fold ? 1 : 0;
        p.flags = d->flags_dev;
        p.scratch = d->gemv;
        return b2::gemv::launch(p, d->stream, d->sm_count, nullptr);
    }
    b2::gemm::Params p = {};
    p.M = (int)a->m; p.N = (int)a->n; p.K = (int)a->k;
    p.bias = out_mode == b2::gemm::OUT_FINAL ? bias : nullptr;
    p.y = static_cast<__half *>(y); p.ldy = (long long)ldy;
    p.partial = a->partial; p.ldp = (long long)a->ldp;
    p.out_mode = out_mode; p.post = a->post; p.fold = fold ? 1 : 0;
    p.vec_y = y && aligned16(y) && ldy % 8 == 0;
    p.vec_p = a->partial && aligned16(a->partial) && a->ldp % 4 == 0;
    p.flags = d->flags_dev;
    if (extra) {
        p.res = static_cast<const __half *>(a->res); p.ldr = (long long)a->ldr;
        p.vec_r = a->res && aligned16(a->res) && a->ldr % 8 == 0;
        p.gate = a->gate; p.gate_n = (int)a->gate_n;
        p.bias2 = static_cast<const __half *>(a->bias2);
        p.gate_table = d->gate_table;
    }
    b2::gemm::Shape s = {a->x, a->ldx, a->w, a->ldw};
    return b2::gemm::launch(s, p, d->stream, d->ordinal, d->sm_count, nullptr);
}

// Kernels launch_core issues for `a`: one GEMM, or the small-M launches (row groups when the x rows
// exceed the streamed kernel's table).
static unsigned core_launches(const b2k_linear *a) {
    if (!use_gemv(a)) return 1;
    const int n = b2::gemv::stream_launches((int)a->m, (int)a->n, (int)a->k, (long long)a->ldw);
    return n > 0 ? (unsigned)n : 1u;
}

static bool fp16_operand_ok(const void *p, size_t ld, size_t cols) {
    return p && aligned16(p) && ld % 8 == 0 && ld >= cols;
}

// The packed gate|up Linear: fused in the GEMM's epilogue, else folded sums to tmp + combine.
static int linear_gated(b2_dev *d, const b2k_linear *a, unsigned *launches) {
    const size_t h32 = ((size_t)a->gate_n + 31) / 32 * 32;
    if ((a->gate != b2::GATE_SIGMOID && a->gate != b2::GATE_GELU) || a->acc != 0 || a->post || a->res ||
        a->raw_only || !a->gate_n || a->n != 2 * h32 || !a->y || a->ldy < a->gate_n)
        return ROCKET_E_SHAPE;
    if (a->fused && !use_gemv(a)) {
        const cudaError_t e = launch_core(d, a, b2::gemm::OUT_FINAL, true, a->y, a->ldy, true);
        if (e != cudaSuccess) return rc_of(e);
        *launches = 1;
        return 0;
    }
    if (!fp16_operand_ok(a->tmp, a->ldt, a->n) || !fp16_operand_ok(a->y, a->ldy, a->gate_n)) return ROCKET_E_SHAPE;
    cudaError_t e = launch_core(d, a, b2::gemm::OUT_RAW16, true, a->tmp, a->ldt, false);
    if (e != cudaSuccess) return rc_of(e);
    *launches = core_launches(a);
    b2::graph::GatedParams g = {};
    g.rows = (int)a->m; g.gate_n = (int)a->gate_n; g.act = a->gate;
    g.src = static_cast<const __half *>(a->tmp); g.lds = (long long)a->ldt;
    g.bias_gate = static_cast<const __half *>(a->bias);
    g.bias_up = static_cast<const __half *>(a->bias2);
    g.y = static_cast<__half *>(a->y); g.ldy = (long long)a->ldy;
    g.gate_table = d->gate_table;
    g.flags = d->flags_dev;
    e = b2::graph::gated_combine(g, d->stream, d->sm_count);
    if (e != cudaSuccess) return rc_of(e);
    *launches += 1;
    return 0;
}

int b2d_linear(b2_dev *d, const b2k_linear *a, unsigned *launches) {
    *launches = 0;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!linear_args_ok(a)) return ROCKET_E_SHAPE;
    if (a->gate) return linear_gated(d, a, launches);
    const bool fold = a->acc == 0 && !a->raw_only;
    int out_mode;
    if (a->raw_only) out_mode = b2::gemm::OUT_RAW32;
    else if (a->fused) out_mode = b2::gemm::OUT_FINAL;
    else out_mode = fold ? b2::gemm::OUT_RAW16 : b2::gemm::OUT_RAW32;
    if (out_mode == b2::gemm::OUT_RAW32 && (!a->partial || a->ldp < a->n)) return ROCKET_E_SHAPE;
    if (out_mode != b2::gemm::OUT_RAW32 && (!a->y || a->ldy < a->n)) return ROCKET_E_SHAPE;
    if (a->res && (a->raw_only || !fp16_operand_ok(a->res, a->ldr, a->n) || !fp16_operand_ok(a->y, a->ldy, a->n)))
        return ROCKET_E_SHAPE;
    const bool fuse_res = a->res && a->fused && !use_gemv(a);
    cudaError_t e = launch_core(d, a, out_mode, fold, a->y, a->ldy, fuse_res);
    if (e != cudaSuccess) return rc_of(e);
    *launches = core_launches(a);
    if (!a->fused && !a->raw_only) {
        // Separate epilogue: FP32 partial -> y, or the folded FP16 sum in y -> y in place.
        b2::aux::EpilogueParams ep = {};
        ep.M = (int)a->m; ep.N = (int)a->n;
        ep.partial = fold ? nullptr : a->partial; ep.ldp = (long long)a->ldp;
        ep.bias = static_cast<const __half *>(a->bias);
        ep.y = static_cast<__half *>(a->y); ep.ldy = (long long)a->ldy;
        ep.post = a->post;
        ep.flags = d->flags_dev;
        e = b2::aux::epilogue(ep, d->stream, d->sm_count);
        if (e != cudaSuccess) return rc_of(e);
        *launches += 1;
    }
    if (a->res && !fuse_res) {
        b2::graph::EwParams ew = {};
        ew.op = b2::graph::EW_ADD; ew.rows = (int)a->m; ew.cols = (int)a->n;
        ew.a = static_cast<const __half *>(a->y); ew.lda = (long long)a->ldy;
        ew.b = static_cast<const __half *>(a->res); ew.ldb = (long long)a->ldr;
        ew.y = static_cast<__half *>(a->y); ew.ldy = (long long)a->ldy;
        ew.flags = d->flags_dev;
        e = b2::graph::elementwise(ew, d->stream, d->sm_count);
        if (e != cudaSuccess) return rc_of(e);
        *launches += 1;
    }
    return 0;
}

int b2d_linear_cube(b2_dev *d, const b2k_linear *a, const b2k_cube_io *io, unsigned *launches) {
    *launches = 0;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!a || !io || !io->in || !io->out || !a->w || a->ldw % 8 || !aligned16(a->w) || a->ldw < a->k)
        return ROCKET_E_SHAPE;
    if (a->m <= B2D_GEMV_MAX_M || !a->fused || a->raw_only || a->res || a->gate || !io->kviews || !io->ntiles ||
        io->nin > B2D_CUBE_MAX_VIEWS || io->nout > B2D_CUBE_MAX_VIEWS || io->nin % io->kviews ||
        io->nout % io->ntiles || io->kview_k % b2::gemm::TILE_K)
        return ROCKET_E_UNSUPPORTED;
    constexpr size_t MAPS = B2D_CUBE_MAX_VIEWS * sizeof(CUtensorMap);
    constexpr size_t OUTS = B2D_CUBE_MAX_VIEWS * sizeof(b2::gemm::CubeOut);
    constexpr size_t BYTES = MAPS + OUTS + B2D_CUBE_MAX_VIEWS;   // + one octet flag per map
    if (!d->cube_dev) {
        if (cudaMalloc(&d->cube_dev, BYTES) != cudaSuccess) {
            cudaGetLastError();
            d->cube_dev = nullptr;
            return ROCKET_E_NOMEM;
        }
    }
    if (!d->cube_host) {
        if (cudaHostAlloc(&d->cube_host, BYTES, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            d->cube_host = nullptr;
            return ROCKET_E_NOMEM;
        }
    }
    if (!d->cube_key) {
        d->cube_key = static_cast<b2k_cube_tile *>(calloc(B2D_CUBE_MAX_VIEWS, sizeof(b2k_cube_tile)));
        if (!d->cube_key) return ROCKET_E_NOMEM;
    }
    // The tables of the previous call stay on the device: a map or an output entry is re-encoded and
    // the tables copied again only when a view differs (callers typically reuse their views, and
    // encoding 256 maps costs more host time than the GEMM).
    CUtensorMap *maps = static_cast<CUtensorMap *>(d->cube_host);
    b2::gemm::CubeOut *outs = reinterpret_cast<b2::gemm::CubeOut *>(static_cast<char *>(d->cube_host) + MAPS);
    unsigned char *octs = static_cast<unsigned char *>(d->cube_host) + MAPS + OUTS;
    bool same_in = io->nin <= d->cube_maps, same_out = io->nout <= d->cube_outs;
    for (unsigned i = 0; same_in && i < io->nin; ++i) {
        const b2k_cube_tile &t = io->in[i], &k = d->cube_key[i];
        same_in = t.ptr == k.ptr && t.rows == k.rows && t.cols == k.cols && t.physical_rows == k.physical_rows;
    }
    for (unsigned i = 0; same_out && i < io->nout; ++i) {
        const b2k_cube_tile &t = io->out[i];
        const b2::gemm::CubeOut &o = outs[i];
        same_out = o.ptr == t.ptr && o.prow == (int)t.physical_rows && o.rows == (int)t.rows && o.cols == (int)t.cols &&
                   o.pcols == (int)t.physical_cols;
    }
    if (!same_in || !same_out) {
        // the staging is rewritten only once the previous cube launch's copy of it has completed
        if (cudaStreamSynchronize(d->stream) != cudaSuccess) return ROCKET_E_DEVICE;
        d->cube_maps = d->cube_outs = 0;   // the device copy is stale until the copies below are queued
    }
    if (!same_in) {
        for (unsigned i = 0; i < io->nin; ++i) {
            const b2k_cube_tile &t = io->in[i];
            int oct = 0;
            if (t.cols % 8 || !b2::gemm::make_cube_map(&maps[i], t.ptr, t.rows, t.physical_rows, t.cols, &oct))
                return ROCKET_E_UNSUPPORTED;
            octs[i] = (unsigned char)oct;
            d->cube_key[i] = t;
        }
    }
    if (!same_out) {
        for (unsigned i = 0; i < io->nout; ++i) {
            const b2k_cube_tile &t = io->out[i];
            if (!aligned16(t.ptr) || t.physical_rows < t.rows || t.physical_cols < t.cols || t.physical_cols % 8)
                return ROCKET_E_UNSUPPORTED;
            outs[i] = b2::gemm::CubeOut{static_cast<__half *>(t.ptr), (int)t.physical_rows, (int)t.rows,
                                        (int)t.cols, (int)t.physical_cols, {0, 0}};
        }
    }
    if (!same_in || !same_out) {
        // both tables again (the other one was left stale above)
        cudaError_t e = cudaMemcpyAsync(d->cube_dev, d->cube_host, io->nin * sizeof(CUtensorMap),
                                        cudaMemcpyHostToDevice, d->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<char *>(d->cube_dev) + MAPS + OUTS, octs, io->nin, cudaMemcpyHostToDevice,
                                d->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<char *>(d->cube_dev) + MAPS, outs, io->nout * sizeof(b2::gemm::CubeOut),
                                cudaMemcpyHostToDevice, d->stream);
        if (e != cudaSuccess) return rc_of(e);
        d->cube_maps = io->nin;
        d->cube_outs = io->nout;
    }
    cudaError_t e;
    b2::gemm::Params p = {};
    p.M = (int)a->m; p.N = (int)a->n; p.K = (int)a->k;
    p.bias = static_cast<const __half *>(a->bias);
    p.out_mode = b2::gemm::OUT_FINAL;
    p.post = a->post;
    p.fold = a->acc == 0 ? 1 : 0;
    p.flags = d->flags_dev;
    p.a_maps = static_cast<const CUtensorMap *>(d->cube_dev);
    p.a_octets = static_cast<const unsigned char *>(d->cube_dev) + MAPS + OUTS;
    p.a_kviews = (int)io->kviews;
    p.a_kview_k = (int)io->kview_k;
    p.y_cube = reinterpret_cast<const b2::gemm::CubeOut *>(static_cast<const char *>(d->cube_dev) + MAPS);
    p.y_cube_nt = (int)io->ntiles;
    b2::gemm::Shape s = {nullptr, 0, a->w, a->ldw};
    e = b2::gemm::launch(s, p, d->stream, d->ordinal, d->sm_count, nullptr);
    if (e != cudaSuccess) return rc_of(e);
    *launches = 1;
    return 0;
}

int b2d_linear_group(b2_dev *d, const b2k_linear *ops, unsigned count, unsigned *launches) {
    *launches = 0;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!ops || !count || count > B2D_GROUP_MAX) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < count; ++i) {
        const b2k_linear *a = &ops[i];
        if (!linear_args_ok(a) || a->m != ops[0].m || !a->fused || a->raw_only || !a->y || a->ldy < a->n)
            return ROCKET_E_SHAPE;
    }
    b2::gemv::Group g = {};
    g.M = (int)ops[0].m;
    g.flags = d->flags_dev;
    g.scratch = d->gemv;
    for (unsigned i = 0; i < count; ++i) {
        const b2k_linear *a = &ops[i];
        if (!b2::gemv::streamed((int)a->m, (int)a->n, (int)a->k, (long long)a->ldw)) continue;
        g.prob[g.count++] = b2::gemv::Problem{static_cast<const __half *>(a->x), (long long)a->ldx,
                                              static_cast<const __half *>(a->w), (long long)a->ldw,
                                              static_cast<const __half *>(a->bias), static_cast<__half *>(a->y),
                                              (long long)a->ldy, nullptr, 0, (int)a->n, (int)a->k,
                                              b2::gemv::OUT_FINAL, a->post, a->acc == 0 ? 1 : 0, 0, 0, 0, 0};
    }
    if (g.count) {
        unsigned l = 0;
        const cudaError_t e = b2::gemv::launch_group(g, d->stream, d->sm_count, nullptr, &l);
        *launches = l;
        if (e != cudaSuccess) return rc_of(e);
    }
    for (unsigned i = 0; i < count; ++i) {
        if (b2::gemv::streamed((int)ops[i].m, (int)ops[i].n, (int)ops[i].k, (long long)ops[i].ldw)) continue;
        unsigned l = 0;
        const int rc = b2d_linear(d, &ops[i], &l);
        *launches += l;
        if (rc) return rc;
    }
    return 0;
}

int b2d_ipc_export(b2_dev *d, const void *ptr, unsigned char out[B2D_IPC_HANDLE_BYTES]) {
    if (!set_device(d) || !ptr || !out) return ROCKET_E_SHAPE;
    static_assert(sizeof(cudaIpcMemHandle_t) == B2D_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(ptr));
    if (e != cudaSuccess) return rc_of(e);
    memcpy(out, &h, sizeof(h));
    return 0;
}

int b2d_ipc_open(b2_dev *d, const unsigned char in[B2D_IPC_HANDLE_BYTES], void **ptr) {
    if (!set_device(d) || !in || !ptr) return ROCKET_E_SHAPE;
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, in, sizeof(h));
    return rc_of(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int b2d_ipc_close(b2_dev *d, void *ptr) {
    if (!set_device(d) || !ptr) return ROCKET_E_SHAPE;
    return rc_of(cudaIpcCloseMemHandle(ptr));
}

struct b2_timer {
    int ordinal;
    cudaEvent_t ev[B2D_TIMER_MARKS];
};

int b2d_timer_create(b2_dev *d, b2_timer **out) {
    *out = nullptr;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    b2_timer *t = static_cast<b2_timer *>(calloc(1, sizeof(b2_timer)));
    if (!t) return ROCKET_E_NOMEM;
    t->ordinal = d->ordinal;
    for (unsigned i = 0; i < B2D_TIMER_MARKS; ++i)
        if (cudaEventCreate(&t->ev[i]) != cudaSuccess) {
            cudaGetLastError();
            b2d_timer_destroy(t);
            return ROCKET_E_DEVICE;
        }
    *out = t;
    return 0;
}

void b2d_timer_destroy(b2_timer *t) {
    if (!t) return;
    cudaSetDevice(t->ordinal);
    for (unsigned i = 0; i < B2D_TIMER_MARKS; ++i)
        if (t->ev[i]) cudaEventDestroy(t->ev[i]);
    free(t);
}

int b2d_timer_mark(b2_dev *d, b2_timer *t, unsigned mark) {
    if (!t || mark >= B2D_TIMER_MARKS || !set_device(d)) return ROCKET_E_SHAPE;
    return rc_of(cudaEventRecord(t->ev[mark], d->stream));
}

int b2d_timer_ms(b2_timer *t, unsigned from, unsigned to, float *ms) {
    if (!t || !ms || from >= B2D_TIMER_MARKS || to >= B2D_TIMER_MARKS) return ROCKET_E_SHAPE;
    cudaSetDevice(t->ordinal);
    cudaError_t e = cudaEventSynchronize(t->ev[to]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, t->ev[from], t->ev[to]);
    if (e != cudaSuccess) cudaGetLastError();
    return e == cudaSuccess ? 0 : ROCKET_E_DEVICE;
}

int b2d_ksplit_round(b2_dev *d, const b2k_linear *a, const b2k_ksplit *ks, unsigned *launches) {
    *launches = 0;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!a || !ks || !linear_args_ok(a) || a->m <= B2D_GEMV_MAX_M || ks->world < 1 ||
        ks->world > (unsigned)b2::ksplit::MAX_WORLD || ks->rank >= ks->world || !ks->rows_per_rank ||
        ks->rows_per_rank % 32 ||
        a->m > ks->world * ks->rows_per_rank || ks->ldp < a->n || ks->ldp % 4 || ks->own_rows > ks->rows_per_rank ||
        (ks->own_rows && (!ks->y_own || ks->ldy < a->n)))
        return ROCKET_E_SHAPE;
    for (unsigned q = 0; q < ks->world; ++q)
        if (!ks->bufs[q]) return ROCKET_E_SHAPE;
    using namespace b2::ksplit;
    const size_t slot = (size_t)ks->rows_per_rank * ks->ldp;
    const long long plane = (long long)(slot * ks->world);
    auto planes_of = [&](unsigned q) {
        return reinterpret_cast<float *>(static_cast<char *>(ks->bufs[q]) + PLANES_OFFSET);
    };
    char *mine = static_cast<char *>(ks->bufs[ks->rank]);
    unsigned *seq = reinterpret_cast<unsigned *>(mine + SEQ_OFFSET);

    // 1. GEMM, raw FP32, row block q routed to rank q's slot for this rank
    b2::gemm::Params p = {};
    p.M = (int)a->m; p.N = (int)a->n; p.K = (int)a->k;
    p.ldp = (long long)ks->ldp;
    p.out_mode = b2::gemm::OUT_RAW32;
    p.vec_p = 1;
    p.flags = d->flags_dev;
    for (unsigned q = 0; q < ks->world; ++q) p.route_dst[q] = planes_of(q) + ks->rank * slot;
    p.route_plane = plane;
    p.route_seq = seq;
    p.route_rows = (int)ks->rows_per_rank;
    p.partial = p.route_dst[ks->rank];
    b2::gemm::Shape s = {a->x, a->ldx, a->w, a->ldw};
    if (ks->timer && cudaEventRecord(ks->timer->ev[0], d->stream) != cudaSuccess) return ROCKET_E_DEVICE;
    cudaError_t e = b2::gemm::launch(s, p, d->stream, d->ordinal, d->sm_count, nullptr);
    if (e != cudaSuccess) return rc_of(e);
    *launches = 1;
    if (ks->timer && cudaEventRecord(ks->timer->ev[1], d->stream) != cudaSuccess) return ROCKET_E_DEVICE;

    // 2. round signal
    SignalParams sp = {};
    sp.seq = seq;
    sp.world = (int)ks->world;
    for (unsigned q = 0; q < ks->world; ++q)
        sp.peer_flag[q] = reinterpret_cast<unsigned *>(static_cast<char *>(ks->bufs[q]) + FLAGS_OFFSET) + ks->rank;
    if ((e = b2::ksplit::signal(sp, d->stream)) != cudaSuccess) return rc_of(e);
    *launches = 2;
    if (ks->timer && cudaEventRecord(ks->timer->ev[2], d->stream) != cudaSuccess) return ROCKET_E_DEVICE;

    // 3. reduction of the owned rows
    ReduceParams rp = {};
    rp.seq = seq;
    rp.flags = reinterpret_cast<const unsigned *>(mine + FLAGS_OFFSET);
    rp.planes = planes_of(ks->rank);
    rp.plane_floats = plane;
    rp.world = (int)ks->world;
    rp.rows_per_rank = (int)ks->rows_per_rank;
    rp.rows = (int)ks->own_rows;
    rp.n = (int)a->n;
    rp.ldp = (long long)ks->ldp;
    rp.vec = ks->own_rows ? (aligned16(ks->y_own) && ks->ldy % 8 == 0) : 0;
    rp.bias = static_cast<const __half *>(ks->bias);
    rp.post = ks->post;
    rp.y = static_cast<__half *>(ks->y_own);
    rp.ldy = (long long)ks->ldy;
    rp.status = d->flags_dev;
    if ((e = b2::ksplit::reduce(rp, d->stream, d->sm_count)) != cudaSuccess) return rc_of(e);
    if (ks->timer && cudaEventRecord(ks->timer->ev[3], d->stream) != cudaSuccess) return ROCKET_E_DEVICE;
    *launches = ks->own_rows ? 3 : 2;
    return 0;
}

int b2d_epilogue(b2_dev *d, unsigned m, unsigned n, const float *partial, size_t ldp, const void *bias, int post,
                 int acc, void *y, size_t ldy) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!m || !n || !partial || !y || ldp < n || ldy < n || acc != 1) return ROCKET_E_SHAPE;
    b2::aux::EpilogueParams ep = {};
    ep.M = (int)m; ep.N = (int)n;
    ep.partial = partial; ep.ldp = (long long)ldp;
    ep.bias = static_cast<const __half *>(bias);
    ep.y = static_cast<__half *>(y); ep.ldy = (long long)ldy;
    ep.post = post;
    ep.flags = d->flags_dev;
    return rc_of(b2::aux::epilogue(ep, d->stream, d->sm_count));
}

int b2d_scan_nonfinite(b2_dev *d, const void *p, size_t rows, size_t cols, size_t ld, uint32_t bit) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    const int flag = flag_of_bit(bit);
    if (flag < 0 || !p || ld % 8 || !aligned16(p)) return ROCKET_E_SHAPE;
    if (!rows || !cols) return 0;
    return rc_of(b2::aux::scan_nonfinite(p, rows, cols, ld, d->flags_dev, flag, d->stream, d->sm_count));
}

static bool to_tiles(const b2k_cube_tile *in, unsigned count, b2::aux::CubeTiles *t) {
    if (count > b2::aux::MAX_TILES) return false;
    memset(t, 0, sizeof(*t));
    for (unsigned i = 0; i < count; ++i) {
        if (!in[i].ptr || !aligned16(in[i].ptr) || in[i].physical_cols % 8 || in[i].rows > in[i].physical_rows ||
            in[i].cols > in[i].physical_cols)
            return false;
        t->tile[i] = {in[i].ptr, in[i].rows, in[i].cols, in[i].physical_rows, in[i].physical_cols, in[i].row0,
                      in[i].col0};
    }
    t->count = count;
    return true;
}

int b2d_cube_to_rowmajor(b2_dev *d, const b2k_cube_tile *tiles, unsigned count, void *dst, size_t ld) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    b2::aux::CubeTiles t;
    if (!to_tiles(tiles, count, &t) || !dst || !aligned16(dst) || ld % 8) return ROCKET_E_SHAPE;
    return rc_of(b2::aux::cube_gather(t, dst, ld, d->stream, d->sm_count));
}

int b2d_rowmajor_to_cube(b2_dev *d, const void *src, size_t ld, const b2k_cube_tile *tiles, unsigned count) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    b2::aux::CubeTiles t;
    if (!to_tiles(tiles, count, &t) || !src || !aligned16(src) || ld % 8) return ROCKET_E_SHAPE;
    return rc_of(b2::aux::cube_scatter(src, ld, t, d->stream, d->sm_count));
}

int b2d_guard_init(b2_dev *d, void *base, size_t payload, size_t slack, size_t guard) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    return rc_of(cudaMemsetAsync(static_cast<char *>(base) + payload + slack, 0xa5, guard, d->stream));
}

int b2d_guard_check(b2_dev *d, void *const *bases, const size_t *payloads, unsigned count, size_t slack,
                    size_t guard) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (count > b2::aux::MAX_TILES) return ROCKET_E_SHAPE;
    b2::aux::GuardList g;
    memset(&g, 0, sizeof(g));
    for (unsigned i = 0; i < count; ++i) {
        g.base[i] = bases[i];
        g.payload[i] = payloads[i];
    }
    g.count = count;
    return rc_of(b2::aux::guard_check(g, slack, guard, d->flags_dev, d->stream));
}

// ----------------------------------------------------------------------------- plan (RKPlan) tiles
}  // extern "C"

namespace {

// The geometry rules every plan view satisfies (the plan verifier enforces them first; the kernels
// index by them, so they are checked again before any launch).
bool rk_tile_ok(const b2k_rk_tile &t) {
    if (!t.ptr || (reinterpret_cast<uintptr_t>(t.ptr) & 15) || !t.rows || !t.cols || t.rows > t.physical_rows ||
        t.cols > t.physical_cols || t.physical_cols > 65520u || t.physical_rows > 4096u)
        return false;
    if (t.layout == B2K_RK_LINEAR) return t.physical_rows == 1;
    if (t.layout == B2K_RK_WEIGHT) return t.physical_rows % 32 == 0 && t.physical_cols % 32 == 0;
    return t.layout == B2K_RK_CUBE && t.physical_rows % 4 == 0 && t.physical_cols % 32 == 0 &&
           t.physical_rows <= 256;
}

bool rk_same_geometry(const b2k_rk_tile &a, const b2k_rk_tile &b) {
    return a.layout == b.layout && a.physical_rows == b.physical_rows && a.physical_cols == b.physical_cols;
}

}  // namespace

extern "C" {

int b2d_rk_pack(b2_dev *d, const b2k_rk_pack *items, unsigned count) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (count && !items) return ROCKET_E_SHAPE;
    for (unsigned base = 0; base < count; base += B2K_RK_MAX_PACK) {
        b2::rkplan::PackTable t;
        memset(&t, 0, sizeof(t));
        size_t max_vectors = 0;
        for (unsigned i = base; i < count && i - base < B2K_RK_MAX_PACK; ++i) {
            const b2k_rk_pack &it = items[i];
            if (!rk_tile_ok(it.dst) || it.mode > B2K_RK_SRC_CHANNEL || (it.rows && it.cols && !it.src) ||
                (size_t)it.r0 + it.rows > it.dst.physical_rows || (size_t)it.c0 + it.cols > it.dst.physical_cols ||
                (it.mode == B2K_RK_SRC_MATRIX && it.rows && it.cols && it.ld < (it.transpose ? it.rows : it.cols)))
                return ROCKET_E_SHAPE;
            t.item[t.count++] = it;
            const size_t v = ((size_t)it.dst.physical_rows * it.dst.physical_cols + 7) / 8;
            if (v > max_vectors) max_vectors = v;
        }
        const int rc = rc_of(b2::rkplan::pack(t, max_vectors, d->stream, d->sm_count));
        if (rc) return rc;
    }
    return 0;
}

int b2d_rk_task(b2_dev *d, const b2k_rk_task *t) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!t || !rk_tile_ok(t->x) || !rk_tile_ok(t->y)) return ROCKET_E_SHAPE;
    const unsigned op = t->op;
    if ((op >= 5 && op <= 7) || op == 10) {
        if (!rk_same_geometry(t->x, t->y)) return ROCKET_E_SHAPE;
    } else if (op >= 1 && op <= 9) {
        if (t->x.layout != B2K_RK_CUBE || !rk_tile_ok(t->w) || t->w.layout != B2K_RK_WEIGHT ||
            t->y.layout != B2K_RK_CUBE || t->x.physical_cols > 256 || t->w.physical_cols != t->x.physical_cols ||
            t->w.physical_rows < t->y.physical_cols || t->y.physical_rows > t->x.physical_rows)
            return ROCKET_E_SHAPE;
        if (op != 1 && (!rk_tile_ok(t->aux) || !rk_same_geometry(t->aux, t->y))) return ROCKET_E_SHAPE;
    } else {
        return ROCKET_E_SHAPE;
    }
    return rc_of(b2::rkplan::task(*t, d->stream, d->sm_count));
}

int b2d_rk_chain(b2_dev *d, const b2k_rk_chain *t) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (!t || !t->n || t->n > B2K_RK_CHAIN_MAX || (t->n < 2 && !t->lut) || !t->scratch || !t->tickets ||
        !rk_tile_ok(t->y) || t->y.layout != B2K_RK_CUBE)
        return ROCKET_E_SHAPE;
    if (t->lut && !((t->lut >= 5 && t->lut <= 7) || t->lut == 10)) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < t->n; ++i) {
        const b2k_rk_tile &x = t->x[i], &w = t->w[i];
        if (!rk_tile_ok(x) || x.layout != B2K_RK_CUBE || !rk_tile_ok(w) || w.layout != B2K_RK_WEIGHT ||
            x.physical_cols > 256 || w.physical_cols != x.physical_cols || w.physical_rows < t->y.physical_cols ||
            t->y.physical_rows > x.physical_rows)
            return ROCKET_E_SHAPE;
    }
    return rc_of(b2::rkplan::chain(*t, d->stream));
}

int b2d_rk_unpack(b2_dev *d, const b2k_rk_unpack *items, unsigned count) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (count && !items) return ROCKET_E_SHAPE;
    for (unsigned base = 0; base < count; base += B2K_RK_MAX_UNPACK) {
        b2::rkplan::UnpackTable t;
        memset(&t, 0, sizeof(t));
        size_t max_elements = 0;
        for (unsigned i = base; i < count && i - base < B2K_RK_MAX_UNPACK; ++i) {
            const b2k_rk_unpack &it = items[i];
            if (!rk_tile_ok(it.src) || !it.dst || it.ld < it.src.cols) return ROCKET_E_SHAPE;
            t.item[t.count++] = it;
            const size_t n = (size_t)it.src.rows * it.src.cols;
            if (n > max_elements) max_elements = n;
        }
        const int rc = rc_of(b2::rkplan::unpack(t, max_elements, d->stream, d->sm_count));
        if (rc) return rc;
    }
    return 0;
}

// ----------------------------------------------------------------------------- graph node kernels
int b2d_elementwise(b2_dev *d, int op, unsigned rows, unsigned cols, const void *a, size_t lda, const void *b,
                    size_t ldb, void *y, size_t ldy) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    const bool binary = op == B2D_EW_ADD || op == B2D_EW_MUL;
    if (op < B2D_EW_ADD || op > B2D_EW_HSIG || rows > (1u << 24) || cols > (1u << 24) ||
        !fp16_operand_ok(a, lda, cols) || !fp16_operand_ok(y, ldy, cols) || (binary && !fp16_operand_ok(b, ldb, cols)))
        return ROCKET_E_SHAPE;
    b2::graph::EwParams p = {};
    p.op = op; p.rows = (int)rows; p.cols = (int)cols;
    p.a = static_cast<const __half *>(a); p.lda = (long long)lda;
    p.b = static_cast<const __half *>(b); p.ldb = (long long)ldb;
    p.y = static_cast<__half *>(y); p.ldy = (long long)ldy;
    p.gate_table = d->gate_table;
    p.flags = d->flags_dev;
    return rc_of(b2::graph::elementwise(p, d->stream, d->sm_count));
}

int b2d_rmsnorm(b2_dev *d, unsigned rows, unsigned cols, const void *x, size_t ldx, const void *gamma, float eps,
                void *y, size_t ldy) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    if (rows > (1u << 24) || cols > (1u << 24) || !gamma || !(eps > 0.0f) || !fp16_operand_ok(x, ldx, cols) ||
        !fp16_operand_ok(y, ldy, cols))
        return ROCKET_E_SHAPE;
    b2::graph::NormParams p = {};
    p.rows = (int)rows; p.cols = (int)cols;
    p.x = static_cast<const __half *>(x); p.ldx = (long long)ldx;
    p.gamma = static_cast<const __half *>(gamma); p.eps = eps;
    p.y = static_cast<__half *>(y); p.ldy = (long long)ldy;
    p.flags = d->flags_dev;
    return rc_of(b2::graph::rmsnorm(p, d->stream, d->sm_count));
}

// ----------------------------------------------------------------------------- CUDA graphs
}  // extern "C"

struct b2_exec {
    cudaGraphExec_t exec;
    int ordinal;
};

extern "C" {

int b2d_capture_begin(b2_dev *d) {
    if (!set_device(d)) return ROCKET_E_DEVICE;
    // every launcher's one-time setup happens outside the capture
    if (b2::gemm::prepare(d->ordinal, d->sm_count) != cudaSuccess || b2::gemv::prepare() != cudaSuccess) {
        cudaGetLastError();
        return ROCKET_E_UNSUPPORTED;
    }
    // thread-local: launches from other threads are neither recorded nor blocked
    if (cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return ROCKET_E_UNSUPPORTED;
    }
    return 0;
}

int b2d_capture_end(b2_dev *d, b2_exec **out, unsigned *kernels) {
    *out = nullptr;
    if (kernels) *kernels = 0;
    if (!set_device(d)) return ROCKET_E_DEVICE;
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(d->stream, &graph);
    if (e != cudaSuccess || !graph) {
        cudaGetLastError();
        if (graph) cudaGraphDestroy(graph);
        return ROCKET_E_DEVICE;
    }
    size_t nodes = 0;
    cudaGraphGetNodes(graph, nullptr, &nodes);
    b2_exec *x = new (std::nothrow) b2_exec();
    if (!x) {
        cudaGraphDestroy(graph);
        return ROCKET_E_NOMEM;
    }
    x->ordinal = d->ordinal;
    const cudaError_t ie = cudaGraphInstantiate(&x->exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
        cudaGetLastError();
        delete x;
        return rc_of(ie);
    }
    if (kernels) *kernels = (unsigned)nodes;
    *out = x;
    return 0;
}

int b2d_exec_launch(b2_dev *d, b2_exec *x) {
    if (!set_device(d) || !x) return ROCKET_E_SHAPE;
    if (x->ordinal != d->ordinal) return ROCKET_E_SHAPE;
    return rc_of(cudaGraphLaunch(x->exec, d->stream));
}

void b2d_exec_destroy(b2_exec *x) {
    if (!x) return;
    cudaSetDevice(x->ordinal);
    cudaGraphExecDestroy(x->exec);
    delete x;
}

}  // extern "C"
