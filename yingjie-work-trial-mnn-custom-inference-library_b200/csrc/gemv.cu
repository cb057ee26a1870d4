// Host side of the W4A16 GEMV: XQ4 reading, B200 row layout, launchers, generic kernel,
// and the kernel-level C ABI entry points for matrices (xq_kernels.h).
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <vector>

#include "../../include/xq_kernels.h"
#include "gemv.hpp"
#include "mma_gemv.hpp"
#include "prefill_gemm.hpp"

namespace xqb {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

// readXq4 (custom_model.cpp:218-262): same header checks, plus size consistency checks the
// reference leaves implicit (its GEMV would read out of bounds on an inconsistent file).
bool read_xq4_file(const std::string& path, HostMatrix* m, std::string* error) {
    std::ifstream in(path, std::ios::binary);
    if (!in) {
        *error = "missing xq4 matrix: " + path;
        return false;
    }
    char magic[8] = {};
    in.read(magic, 8);
    if (!in || std::memcmp(magic, "XQW4A16", 7) != 0) {
        *error = "bad xq4 magic: " + path;
        return false;
    }
    uint32_t h[5] = {};
    uint64_t c[3] = {};
    in.read(reinterpret_cast<char*>(h), sizeof h);
    in.read(reinterpret_cast<char*>(c), sizeof c);
    const uint32_t version = h[0], rows = h[1], cols = h[2], group = h[3], bits = h[4];
    if (!in || (version != 1 && version != 2) || bits != 4 || rows == 0 || cols == 0 || group == 0 ||
        c[1] != c[2]) {
        *error = "invalid xq4 header: " + path;
        return false;
    }
    const uint64_t gpr = (cols + group - 1) / group;
    if (c[0] != static_cast<uint64_t>(rows) * ((cols + 1) / 2) || c[1] != static_cast<uint64_t>(rows) * gpr) {
        *error = "inconsistent xq4 sizes: " + path;
        return false;
    }
    m->rows = static_cast<int>(rows);
    m->cols = static_cast<int>(cols);
    m->group = static_cast<int>(group);
    m->version = static_cast<int>(version);
    m->packed.resize(c[0]);
    m->scales.resize(c[1]);
    m->zeros.resize(c[2]);
    in.read(reinterpret_cast<char*>(m->packed.data()), static_cast<std::streamsize>(c[0]));
    in.read(reinterpret_cast<char*>(m->scales.data()), static_cast<std::streamsize>(c[1] * 4));
    in.read(reinterpret_cast<char*>(m->zeros.data()), static_cast<std::streamsize>(c[2] * 4));
    if (!in) {
        *error = "short xq4 payload: " + path;
        return false;
    }
    return true;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("XQ_PDL");
        return !(e && std::atoi(e) == 0);
    }();
    return on;
}

bool fast_shape(int cols, int group) { return group == 64 && cols >= 1024 && cols % 1024 == 0 && cols <= 16384; }

static bool fp16_exact(float v) {
    const __half h = __float2half_rn(v);
    return __half2float(h) == v;
}

bool upload_matrix(const std::vector<const HostMatrix*>& parts, bool interleave_pairs, DevMatrix* out,
                   std::string* error) {
    *out = DevMatrix();
    if (parts.empty()) {
        *error = "empty matrix list";
        return false;
    }
    const int cols = parts[0]->cols, group = parts[0]->group;
    int rows = 0;
    for (const HostMatrix* p : parts) {
        if (p->cols != cols || p->group != group) {
            *error = "matrices fused into one launch must share cols and group size";
            return false;
        }
        rows += p->rows;
    }
    if (interleave_pairs && (parts.size() != 2 || parts[0]->rows != parts[1]->rows)) {
        *error = "paired matrices must have equal rows";
        return false;
    }
    out->rows = rows;
    out->cols = cols;
    out->group = group;
    out->version = parts[0]->version;
    const int gpr = (cols + group - 1) / group;

    if (!fast_shape(cols, group)) {
        // Generic layout: the reference's own arrays, one version for all parts.
        for (const HostMatrix* p : parts)
            if (p->version != out->version) {
                *error = "mixed xq4 versions in a generic-layout matrix";
                return false;
            }
        std::vector<const HostMatrix*> order(parts.begin(), parts.end());
        std::vector<uint8_t> packed;
        std::vector<float> sc, ze;
        const size_t rb = static_cast<size_t>((cols + 1) / 2);
        auto append_row = [&](const HostMatrix* p, int r) {
            packed.insert(packed.end(), p->packed.begin() + r * rb, p->packed.begin() + (r + 1) * rb);
            sc.insert(sc.end(), p->scales.begin() + static_cast<size_t>(r) * gpr,
                      p->scales.begin() + static_cast<size_t>(r + 1) * gpr);
            ze.insert(ze.end(), p->zeros.begin() + static_cast<size_t>(r) * gpr,
                      p->zeros.begin() + static_cast<size_t>(r + 1) * gpr);
        };
        if (interleave_pairs) {
            for (int r = 0; r < parts[0]->rows; ++r) {
                append_row(parts[0], r);
                append_row(parts[1], r);
            }
        } else {
            for (const HostMatrix* p : parts)
                for (int r = 0; r < p->rows; ++r) append_row(p, r);
        }
        out->kind = 2;
        XQB_CUDA_OK(cudaMalloc(&out->d_packed, packed.size()));
        XQB_CUDA_OK(cudaMalloc(&out->d_scales, sc.size() * 4));
        XQB_CUDA_OK(cudaMalloc(&out->d_zeros, ze.size() * 4));
        XQB_CUDA_OK(cudaMemcpy(out->d_packed, packed.data(), packed.size(), cudaMemcpyHostToDevice));
        XQB_CUDA_OK(cudaMemcpy(out->d_scales, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice));
        XQB_CUDA_OK(cudaMemcpy(out->d_zeros, ze.data(), ze.size() * 4, cudaMemcpyHostToDevice));
        out->bytes = packed.size() + 8 * sc.size();
        return true;
    }

    std::vector<uint8_t> host;
    if (!build_matrix_rows(parts, interleave_pairs, out, &host, error)) return false;
    return upload_matrix_rows(host, out, error);
}

bool build_matrix_rows(const std::vector<const HostMatrix*>& parts, bool interleave_pairs, DevMatrix* out,
                       std::vector<uint8_t>* host_out, std::string* error, bool narrow) {
    const int cols = parts[0]->cols, group = parts[0]->group;
    int rows = 0;
    for (const HostMatrix* p : parts) {
        if (p->cols != cols || p->group != group) {
            *error = "matrices fused into one launch must share cols and group size";
            return false;
        }
        rows += p->rows;
    }
    if (!fast_shape(cols, group) && !(narrow && group == 64 && cols >= 512 && cols % 512 == 0)) {
        *error = "matrix shape has no fused row layout";
        return false;
    }
    if (interleave_pairs && (parts.size() != 2 || parts[0]->rows != parts[1]->rows)) {
        *error = "paired matrices must have equal rows";
        return false;
    }
    const int gpr = (cols + group - 1) / group;
    out->rows = rows;
    out->cols = cols;
    out->group = group;
    out->version = parts[0]->version;
    // Decide the metadata kind for the whole fused matrix.
    bool sym = true;
    for (const HostMatrix* p : parts) {
        if (p->version != 1) sym = false;
        for (size_t i = 0; sym && i < p->scales.size(); ++i)
            if (p->zeros[i] != 8.0f || !fp16_exact(p->scales[i])) sym = false;
    }
    out->kind = sym ? 0 : 1;
    out->meta_offset = cols / 2;
    out->row_stride = cols / 2 + (sym ? 2 : 8) * gpr;  // multiple of 16 since cols % 512 == 0
    std::vector<uint8_t>& host = *host_out;
    host.assign(static_cast<size_t>(rows) * out->row_stride, 0);
    size_t dst_row = 0;
    auto emit = [&](const HostMatrix* p, int r) {
        uint8_t* d = host.data() + dst_row * out->row_stride;
        std::memcpy(d, p->packed.data() + static_cast<size_t>(r) * (cols / 2), cols / 2);
        uint8_t* meta = d + out->meta_offset;
        for (int g = 0; g < gpr; ++g) {
            const float s = p->scales[static_cast<size_t>(r) * gpr + g];
            const float z = p->zeros[static_cast<size_t>(r) * gpr + g];
            if (sym) {
                const __half h = __float2half_rn(s);
                std::memcpy(meta + 2 * g, &h, 2);
            } else {
                // y += s * code_dot + b * x_sum; v1: b = -zero * scale, v2: b = zero
                const float pair[2] = {s, p->version == 2 ? z : -z * s};
                std::memcpy(meta + 8 * g, pair, 8);
            }
        }
        ++dst_row;
    };
    if (interleave_pairs) {
        for (int r = 0; r < parts[0]->rows; ++r) {
            emit(parts[0], r);
            emit(parts[1], r);
        }
    } else {
        for (const HostMatrix* p : parts)
            for (int r = 0; r < p->rows; ++r) emit(p, r);
    }
    return true;
}

bool upload_matrix_rows(const std::vector<uint8_t>& host, DevMatrix* out, std::string* error) {
    (void)error;
    out->bytes = host.size();
    XQB_CUDA_OK(cudaMalloc(&out->d_rows, host.size()));
    XQB_CUDA_OK(cudaMemcpy(out->d_rows, host.data(), host.size(), cudaMemcpyHostToDevice));
    return true;
}

namespace {
struct B200Header {
    char magic[8];  // "XQB200\0\0"
    uint32_t version, kind, rows, cols, group, xq4_version, row_stride, meta_offset;
    uint64_t bytes;
    uint8_t reserved[16];
};
static_assert(sizeof(B200Header) == 64, "packed header");
constexpr char kB200Magic[8] = {'X', 'Q', 'B', '2', '0', '0', '\0', '\0'};
}  // namespace

bool write_b200_file(const std::string& path, const DevMatrix& m, const std::vector<uint8_t>& host,
                     std::string* error) {
    B200Header h = {};
    std::memcpy(h.magic, kB200Magic, 8);
    h.version = 1;
    h.kind = static_cast<uint32_t>(m.kind);
    h.rows = static_cast<uint32_t>(m.rows);
    h.cols = static_cast<uint32_t>(m.cols);
    h.group = static_cast<uint32_t>(m.group);
    h.xq4_version = static_cast<uint32_t>(m.version);
    h.row_stride = static_cast<uint32_t>(m.row_stride);
    h.meta_offset = static_cast<uint32_t>(m.meta_offset);
    h.bytes = host.size();
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    f.write(reinterpret_cast<const char*>(&h), sizeof h);
    f.write(reinterpret_cast<const char*>(host.data()), static_cast<std::streamsize>(host.size()));
    if (!f) {
        *error = "cannot write " + path;
        return false;
    }
    return true;
}

bool read_b200_file(const std::string& path, DevMatrix* m, std::vector<uint8_t>* host, std::string* error) {
    std::ifstream f(path, std::ios::binary);
    B200Header h;
    if (!f.read(reinterpret_cast<char*>(&h), sizeof h) || std::memcmp(h.magic, kB200Magic, 8) != 0 || h.version != 1) {
        *error = "not a packed B200 matrix: " + path;
        return false;
    }
    const uint32_t gpr = h.group ? (h.cols + h.group - 1) / h.group : 0;
    if (h.kind > 1 || !fast_shape(static_cast<int>(h.cols), static_cast<int>(h.group)) ||
        h.meta_offset != h.cols / 2 || h.row_stride != h.cols / 2 + (h.kind == 0 ? 2u : 8u) * gpr ||
        h.bytes != static_cast<uint64_t>(h.rows) * h.row_stride) {
        *error = "inconsistent packed B200 header: " + path;
        return false;
    }
    host->resize(h.bytes);
    if (!f.read(reinterpret_cast<char*>(host->data()), static_cast<std::streamsize>(h.bytes))) {
        *error = "truncated packed B200 matrix: " + path;
        return false;
    }
    *m = DevMatrix();
    m->rows = static_cast<int>(h.rows);
    m->cols = static_cast<int>(h.cols);
    m->group = static_cast<int>(h.group);
    m->version = static_cast<int>(h.xq4_version);
    m->kind = static_cast<int>(h.kind);
    m->row_stride = static_cast<int>(h.row_stride);
    m->meta_offset = static_cast<int>(h.meta_offset);
    return true;
}

void free_matrix(DevMatrix* m) {
    cudaFree(m->d_rows);
    cudaFree(m->d_packed);
    cudaFree(m->d_scales);
    cudaFree(m->d_zeros);
    cudaFree(m->d_tiles);
    *m = DevMatrix();
}

namespace {

struct Shape {
    int block, rows_per_chunk, rpt, stages, smem;
};

// Launch-shape knobs (defaults tuned on B200; the environment overrides exist for sweeps).
struct Tuning {
    int block = kTargetBlock;
    int rpt = 8;
    int blocks_per_sm = 2;
    int evict_first = 1;
    int ring_bytes = kRingBudgetBytes;
};

const Tuning& tuning() {
    static const Tuning t = [] {
        Tuning v;
        if (const char* e = std::getenv("XQ_GEMV_BLOCK")) v.block = std::max(32, std::min(kMaxBlock, std::atoi(e)));
        if (const char* e = std::getenv("XQ_GEMV_RPT")) v.rpt = std::atoi(e) >= 8 ? 8 : 4;
        if (const char* e = std::getenv("XQ_GEMV_BPS")) v.blocks_per_sm = std::max(1, std::min(4, std::atoi(e)));
        if (const char* e = std::getenv("XQ_L2_EVICT_FIRST")) v.evict_first = std::atoi(e) != 0;
        if (const char* e = std::getenv("XQ_GEMV_RING_KB"))
            v.ring_bytes = std::max(16, std::min(200, std::atoi(e))) * 1024;
        return v;
    }();
    return t;
}

}  // namespace

int gemv_evict_first() { return tuning().evict_first; }

namespace {

Shape shape_for(const DevMatrix& m) {
    const Tuning& tu = tuning();
    Shape s{};
    const int team = m.cols / 32;
    const int teams = std::max(1, std::min((kMaxBlock - 32) / team, tu.block / team));
    s.block = teams * team + 32;  // + producer warp
    s.rpt = tu.rpt;
    int r = std::min(s.rpt, std::max(2, kStageTargetBytes / m.row_stride));
    r &= ~1;
    s.rows_per_chunk = std::max(2, r);
    const int stage_bytes = s.rows_per_chunk * m.row_stride;
    s.stages = std::max(2, std::min(kMaxStages, tu.ring_bytes / stage_bytes));
    s.smem = kGemvHeaderBytes + s.stages * stage_bytes;
    return s;
}

template <int META, int PRO, int EPI>
cudaError_t launch_one(const GemvParams& p, dim3 grid, const Shape& s, const LaunchCtx& ctx) {
    if (s.rpt == 8)
        return launch_ex(gemv_w4a16_kernel<META, PRO, EPI, 8>, grid, dim3(s.block), static_cast<size_t>(s.smem),
                         ctx.stream, ctx.pdl, p);
    return launch_ex(gemv_w4a16_kernel<META, PRO, EPI, 4>, grid, dim3(s.block), static_cast<size_t>(s.smem),
                     ctx.stream, ctx.pdl, p);
}

template <int META, int PRO, int EPI>
cudaError_t set_smem() {
    const int bytes = 220 * 1024;  // below the 227 KB opt-in limit, leaving room for static smem
    cudaError_t e = cudaFuncSetAttribute(gemv_w4a16_kernel<META, PRO, EPI, 4>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(gemv_w4a16_kernel<META, PRO, EPI, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                bytes);
}

// The (prologue, epilogue) pairs the runtime and the C ABI use.
#define XQB_GEMV_COMBOS(X)      \
    X(kProPlain, kEpiStore)     \
    X(kProPlain, kEpiResidual)  \
    X(kProPlain, kEpiArgmax)    \
    X(kProRms, kEpiStore)       \
    X(kProRms, kEpiConv)        \
    X(kProRms, kEpiSwiglu)      \
    X(kProRms, kEpiArgmax)      \
    X(kProGatedRms, kEpiResidual)

}  // namespace

bool gemv_init_device() {
#define XQB_SET(PRO, EPI)                                          \
    XQB_CUDA_OK((set_smem<kMetaSym16, PRO, EPI>()));               \
    XQB_CUDA_OK((set_smem<kMetaAff32, PRO, EPI>()));
    XQB_GEMV_COMBOS(XQB_SET)
#undef XQB_SET
    return true;
}

int gemv_grid(const DevMatrix& m, int unit, int num_sms, int max_blocks) {
    int g = std::min(num_sms * tuning().blocks_per_sm, m.rows / unit);
    if (max_blocks > 0) g = std::min(g, max_blocks);
    return std::max(1, g);
}

bool launch_gemv(const DevMatrix& m, int pro, int epi, GemvParams p, int unit, const LaunchCtx& ctx,
                 int max_blocks) {
    if (!m.fast()) {
        set_last_error("launch_gemv: matrix is not in the fused layout");
        return false;
    }
    const Shape s = shape_for(m);
    p.w = m.d_rows;
    p.rows = m.rows;
    p.cols = m.cols;
    p.row_stride = m.row_stride;
    p.meta_offset = m.meta_offset;
    p.rows_per_chunk = s.rows_per_chunk;
    p.stages = s.stages;
    p.unit = unit;
    p.evict_first = tuning().evict_first;
    const dim3 grid(gemv_grid(m, unit, ctx.num_sms, max_blocks));
    cudaError_t e = cudaErrorInvalidValue;
#define XQB_CASE(PRO, EPI)                                                          \
    if (pro == PRO && epi == EPI) {                                                 \
        e = m.kind == 0 ? launch_one<kMetaSym16, PRO, EPI>(p, grid, s, ctx)         \
                        : launch_one<kMetaAff32, PRO, EPI>(p, grid, s, ctx);        \
    }
    XQB_GEMV_COMBOS(XQB_CASE)
#undef XQB_CASE
    if (e != cudaSuccess) {
        set_last_error(std::string("gemv launch failed: ") + cudaGetErrorString(e));
        return false;
    }
    return true;
}

// ------------------------------------------------------------------------------------
// Generic kernel: one warp per row, lanes stride over groups; per group the reference's
// algebra s * (code_dot - zero * x_sum) (v1) or s * code_dot + zero * x_sum (v2).
// ------------------------------------------------------------------------------------
__global__ void gemv_generic_kernel(const uint8_t* packed, const float* scales, const float* zeros, int rows,
                                    int cols, int group, int version, const float* x, float* y) {
    const int warps = blockDim.x >> 5;
    const int row = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int gpr = (cols + group - 1) / group;
    const size_t stride = static_cast<size_t>((cols + 1) / 2);
    const uint8_t* rp = packed + static_cast<size_t>(row) * stride;
    float acc = 0.0f;
    for (int g = lane; g < gpr; g += 32) {
        const int c0 = g * group;
        const int c1 = min(cols, c0 + group);
        float cd = 0.0f, xs = 0.0f;
        for (int c = c0; c < c1; ++c) {
            const uint8_t b = rp[c >> 1];
            const float code = static_cast<float>((c & 1) ? (b >> 4) : (b & 0x0f));
            cd += code * x[c];
            xs += x[c];
        }
        const size_t mi = static_cast<size_t>(row) * gpr + g;
        if (version == 2)
            acc += scales[mi] * cd + zeros[mi] * xs;
        else
            acc += scales[mi] * (cd - zeros[mi] * xs);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

bool launch_gemv_generic(const DevMatrix& m, const float* x, float* y, cudaStream_t stream) {
    const int warps = 8;
    gemv_generic_kernel<<<(m.rows + warps - 1) / warps, warps * 32, 0, stream>>>(
        m.d_packed, m.d_scales, m.d_zeros, m.rows, m.cols, m.group, m.version, x, y);
    XQB_CUDA_OK(cudaGetLastError());
    return true;
}

// Single-block argmax over a vector (lowest index on ties), for the generic layout.
__global__ void argmax_vector_kernel(const float* v, int n, int32_t* idx_out, float* val_out) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    if (threadIdx.x == 0) bi = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) argmax_merge(bv, bi, v[i], i);
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) argmax_merge(bv, bi, sv[w], si[w]);
        *idx_out = bi;
        *val_out = bv;
    }
}

}  // namespace xqb

// ------------------------------------------------------------------------------------
// Kernel-level C ABI (xq_kernels.h)
// ------------------------------------------------------------------------------------
struct xqk_matrix {
    xqb::DevMatrix m;
    int device = 0;
    int num_sms = 148;
    float* part_val = nullptr;  // argmax scratch
    int* part_idx = nullptr;
    unsigned* counter = nullptr;
    unsigned* err = nullptr;
    float* y_tmp = nullptr;  // generic argmax / host path staging
    float* x_tmp = nullptr;
    xqb::MmaMatrix mma;  // tensor-core tile copy, when the layout serves the matrix
};

namespace {
std::mutex g_init_mu;
bool g_inited[64] = {};

bool ensure_device(int device) {
    std::lock_guard<std::mutex> lock(g_init_mu);
    XQB_CUDA_OK(cudaSetDevice(device));
    if (device >= 0 && device < 64 && !g_inited[device]) {
        if (!xqb::gemv_init_device() || !xqb::mma_init_device()) return false;
        g_inited[device] = true;
    }
    return true;
}
}  // namespace

extern "C" {

const char* xqk_last_error(void) { return xqb::last_error(); }

int xqk_matrix_create(const uint8_t* packed, const float* scales, const float* zeros, int rows, int cols,
                      int group_size, int version, int device, xqk_matrix** out) {
    if (!packed || !scales || !zeros || !out || rows <= 0 || cols <= 0 || group_size <= 0 ||
        (version != 1 && version != 2)) {
        xqb::set_last_error("xqk_matrix_create: invalid argument");
        return -1;
    }
    *out = nullptr;
    if (!ensure_device(device)) return -4;
    xqb::HostMatrix h;
    h.rows = rows;
    h.cols = cols;
    h.group = group_size;
    h.version = version;
    const size_t gpr = static_cast<size_t>((cols + group_size - 1) / group_size);
    h.packed.assign(packed, packed + static_cast<size_t>(rows) * ((cols + 1) / 2));
    h.scales.assign(scales, scales + rows * gpr);
    h.zeros.assign(zeros, zeros + rows * gpr);
    auto* m = new xqk_matrix();
    m->device = device;
    cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device);
    std::string err;
    if (!xqb::upload_matrix({&h}, false, &m->m, &err)) {
        xqb::set_last_error(err.empty() ? xqb::last_error() : err);
        delete m;
        return -3;
    }
    if (xqb::mma_eligible(h) && !xqb::build_mma_matrix(h, &m->mma, &err)) {
        xqb::set_last_error(err.empty() ? xqb::last_error() : err);
        xqk_matrix_destroy(m);
        return -4;
    }
    const int nb = m->num_sms;
    if (cudaMalloc(&m->part_val, nb * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&m->part_idx, nb * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&m->counter, sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&m->err, sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&m->y_tmp, static_cast<size_t>(rows) * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&m->x_tmp, static_cast<size_t>(cols) * sizeof(float)) != cudaSuccess ||
        cudaMemset(m->counter, 0, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(m->err, 0, sizeof(unsigned)) != cudaSuccess) {
        xqb::set_last_error("xqk_matrix_create: device allocation failed");
        xqk_matrix_destroy(m);
        return -4;
    }
    *out = m;
    return 0;
}

void xqk_matrix_destroy(xqk_matrix* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    xqb::free_matrix(&m->m);
    xqb::free_mma_matrix(&m->mma);
    cudaFree(m->part_val);
    cudaFree(m->part_idx);
    cudaFree(m->counter);
    cudaFree(m->err);
    cudaFree(m->y_tmp);
    cudaFree(m->x_tmp);
    delete m;
}

int xqk_matrix_info(const xqk_matrix* m, int* rows, int* cols, size_t* device_bytes, int* row_stride,
                    int* layout_kind, int* fast_path) {
    if (!m) return -1;
    if (rows) *rows = m->m.rows;
    if (cols) *cols = m->m.cols;
    if (device_bytes) *device_bytes = m->m.bytes;
    if (row_stride) *row_stride = m->m.row_stride;
    if (layout_kind) *layout_kind = m->m.kind;
    if (fast_path) *fast_path = m->m.fast() ? 1 : 0;
    return 0;
}

int xqk_gemv_w4a16(const xqk_matrix* m, const float* x_dev, float* y_dev, void* stream) {
    if (!m || !x_dev || !y_dev) return -1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!m->m.fast()) return xqb::launch_gemv_generic(m->m, x_dev, y_dev, s) ? 0 : -4;
    xqb::GemvParams p = {};
    p.x = x_dev;
    p.out = y_dev;
    p.err = m->err;
    xqb::LaunchCtx ctx;
    ctx.stream = s;
    ctx.num_sms = m->num_sms;
    ctx.pdl = false;
    return xqb::launch_gemv(m->m, xqb::kProPlain, xqb::kEpiStore, p, 1, ctx) ? 0 : -4;
}

int xqk_gemv_w4a16_mma(const xqk_matrix* m, const float* x_dev, float* y_dev, void* stream) {
    if (!m || !x_dev || !y_dev) return -1;
    if (!m->mma.d_tiles) {
        xqb::set_last_error("xqk_gemv_w4a16_mma: matrix not in the tensor-core layout (needs symmetric xq4 v1, "
                            "group 64, fp16-exact scales, cols a multiple of 512 and of 4096 above 4096)");
        return -2;
    }
    return xqb::launch_mma_gemv(m->mma, x_dev, y_dev, m->err, m->num_sms, static_cast<cudaStream_t>(stream), true)
               ? 0
               : -4;
}

int xqk_gemv_w4a16_mma_f16(const xqk_matrix* m, const void* x_dev, void* y_dev, void* stream) {
    if (!m || !x_dev || !y_dev) return -1;
    if (!m->mma.d_tiles) {
        xqb::set_last_error("xqk_gemv_w4a16_mma_f16: matrix not in the tensor-core layout (needs symmetric xq4 v1, "
                            "group 64, fp16-exact scales, cols a multiple of 512 and of 4096 above 4096)");
        return -2;
    }
    if ((reinterpret_cast<uintptr_t>(x_dev) & 7u) != 0) {
        xqb::set_last_error("xqk_gemv_w4a16_mma_f16: x must be 8-byte aligned");
        return -1;
    }
    return xqb::launch_mma_gemv_f16(m->mma, static_cast<const __half*>(x_dev), static_cast<__half*>(y_dev), m->err,
                                    m->num_sms, static_cast<cudaStream_t>(stream), true)
               ? 0
               : -4;
}

int xqk_prefill_gemm_w4a16(const xqk_matrix* m, const void* x_dev, const void* x_lo_dev, int n_tokens, void* y_dev,
                           int ldy, int out_kind, void* stream) {
    if (!m || !x_dev || !y_dev || n_tokens <= 0) return -1;
    if (cudaSetDevice(m->device) != cudaSuccess) return -4;
    return xqb::launch_prefill_gemm(m->m, static_cast<const __nv_bfloat16*>(x_dev),
                                    static_cast<const __nv_bfloat16*>(x_lo_dev), n_tokens, y_dev, ldy, out_kind, m->err,
                                    m->num_sms, static_cast<cudaStream_t>(stream))
               ? 0
               : -1;
}

int xqk_mma_tiles(const uint8_t* packed, const float* scales, int rows, int cols, uint8_t* out, size_t capacity,
                  size_t* written) {
    if (!packed || !scales || !written || rows <= 0 || cols <= 0 || cols % 128 != 0) {
        xqb::set_last_error("xqk_mma_tiles: invalid argument (cols must be a multiple of 128)");
        return -1;
    }
    const size_t need = static_cast<size_t>((rows + 15) / 16) * (cols / 128) * xqb::kMmaUnitBytes;
    *written = need;
    if (!out || capacity < need) return -5;
    std::vector<uint8_t> t;
    if (!xqb::host_mma_tiles(packed, scales, rows, cols, &t)) return -1;
    std::memcpy(out, t.data(), need);
    return 0;
}

int xqk_gemv_w4a16_host(const xqk_matrix* m, const float* x_host, float* y_host) {
    if (!m || !x_host || !y_host) return -1;
    if (cudaSetDevice(m->device) != cudaSuccess) return -4;
    if (cudaMemcpy(m->x_tmp, x_host, m->m.cols * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) return -4;
    if (xqk_gemv_w4a16(m, m->x_tmp, m->y_tmp, nullptr) != 0) return -4;
    if (cudaMemcpy(y_host, m->y_tmp, m->m.rows * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess) {
        xqb::set_last_error("xqk_gemv_w4a16_host: copy failed");
        return -4;
    }
    return 0;
}

int xqk_gemv_w4a16_argmax(const xqk_matrix* m, const float* x_dev, int32_t* index_dev, float* value_dev,
                          void* stream) {
    if (!m || !x_dev || !index_dev || !value_dev) return -1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!m->m.fast()) {
        if (!xqb::launch_gemv_generic(m->m, x_dev, m->y_tmp, s)) return -4;
        xqb::argmax_vector_kernel<<<1, 1024, 0, s>>>(m->y_tmp, m->m.rows, index_dev, value_dev);
        return cudaGetLastError() == cudaSuccess ? 0 : -4;
    }
    xqb::GemvParams p = {};
    p.x = x_dev;
    p.part_val = m->part_val;
    p.part_idx = m->part_idx;
    p.counter = m->counter;
    p.token_out = index_dev;
    p.value_out = value_dev;
    p.err = m->err;
    xqb::LaunchCtx ctx;
    ctx.stream = s;
    ctx.num_sms = m->num_sms;
    ctx.pdl = false;
    return xqb::launch_gemv(m->m, xqb::kProPlain, xqb::kEpiArgmax, p, 1, ctx, m->num_sms) ? 0 : -4;
}

}  // extern "C"
