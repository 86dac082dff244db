// The reference's C++ FFN interface on B200: every function and class method that
// kernels/gpu/include/heteromega/gpu_ffn.hpp and include/hipkernels/w4a16_gemm_packed.hpp declare
// for the FFN path, implemented over the C ABI of libhmb.so (include/hmb.h). A C++ caller of those
// headers (the model loop's GpuFfnModel::forward at src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2852-2865,
// the GEMV/GEMM dispatch of include/unified_llm_w4a16_hetero/hetero_compute.hpp:16-39) links this file
// and libhmb.so in place of kernels/gpu/src/*.cu and src/hipkernels; the headers compile unchanged with
// shim/hip/hip_runtime.h, which makes hipStream_t a cudaStream_t.
//
// Semantics follow the reference: argument errors raise c10::Error through TORCH_CHECK, a failing
// kernel launch raises std::runtime_error, everything is enqueued on the given stream without
// synchronizing, and per-stream scratch is cached and never freed. Deliberate differences:
//   * no 128-row padding of inputs is needed (padded_rows stays as an API): the kernels guard M;
//   * SiLU*up is fused into the gate/up kernels and gpu_ffn_slice_forward runs hmb_w4a16_ffn, so
//     GpuFfnBuffers::gate_up and x_pad stay empty;
//   * both GemvKernel and both GemmKernel values select the B200 kernels;
//   * residual_norm_bf16 writes the normed rows to gemm_x when `normed` is null: the B200 GEMMs read
//     x directly, so the rows the reference would keep in its prepared-input buffer go where the
//     next GEMM reads them, and GemmInputReuse counts the GEMMs that read that x.
// Prefill attention (sdpa_*) is outside the FFN path and is not provided.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/cuda.h>
#include <heteromega/gpu_ffn.hpp>
#include <hipkernels/w4a16_gemm_packed.hpp>

#include <cstdlib>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <tuple>

#include "hmb.h"

namespace {

void hmb_check(int rc, const char *what) {
    if (rc == HMB_OK) return;
    std::string msg = std::string(what) + ": " + hmb_status_string(rc);
    if (rc == HMB_ERR_CUDA) msg += " (cudaError " + std::to_string(hmb_last_cuda_error()) + ")";
    if (rc == HMB_ERR_ARG || rc == HMB_ERR_ALIGN || rc == HMB_ERR_VALUE || rc == HMB_ERR_UNSUPPORTED) TORCH_CHECK(false, msg);
    throw std::runtime_error(msg);
}

int dtype_code(const torch::Tensor &t) {
    switch (t.scalar_type()) {
    case torch::kBFloat16: return HMB_BF16;
    case torch::kHalf: return HMB_FP16;
    case torch::kFloat: return HMB_FP32;
    default: TORCH_CHECK(false, "heteromega: unsupported dtype ", t.scalar_type());
    }
    return -1;
}

int64_t packed_bytes(int64_t k, int64_t n) { return (k / heteromega::kTileK) * (n / heteromega::kTileN) * heteromega::kTileBytes; }

// Zero-filled device scratch for one kind of call on one stream, grown on demand and kept for the
// life of the process (the kernels leave its counter words zero after every call).
std::mutex g_ws_mutex;
std::map<std::tuple<int, cudaStream_t, int>, torch::Tensor> g_ws;
enum { kWsGemv = 0, kWsFfn = 1 };

torch::Tensor &workspace(const torch::Device &device, cudaStream_t stream, int kind, size_t bytes) {
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    torch::Tensor &buf = g_ws[std::make_tuple(static_cast<int>(device.index()), stream, kind)];
    if (!buf.defined() || static_cast<size_t>(buf.numel()) < bytes) {
        const int64_t size = std::max<int64_t>(static_cast<int64_t>(bytes), buf.defined() ? 2 * buf.numel() : int64_t(1) << 20);
        // The old buffer may still be in use by work enqueued on `stream`; the new one is zeroed on it.
        c10::cuda::CUDAStreamGuard guard(c10::cuda::getStreamFromExternal(stream, device.index()));
        buf = torch::zeros({size}, torch::TensorOptions().dtype(torch::kUInt8).device(device));
    }
    return buf;
}

void check_cuda_tensors(const char *what, std::initializer_list<const torch::Tensor *> ts) {
    const torch::Device dev = (*ts.begin())->device();
    for (const torch::Tensor *t : ts) TORCH_CHECK(t->is_cuda() && t->device() == dev, what, ": all tensors must be CUDA tensors on one device");
}

// Rows x columns view of a tensor whose rows are contiguous (1-D tensors are one row).
int64_t rows_of(const torch::Tensor &t) { return t.dim() == 2 ? t.size(0) : 1; }
int64_t ld_of(const torch::Tensor &t) { return t.dim() == 2 ? t.stride(0) : t.size(-1); }

// The product's packed matmul: the decode GEMV up to 16 rows, the tcgen05 GEMM above when the shape
// allows it, else the GEMV over row chunks.
void linear(torch::Tensor &out, const torch::Tensor &in, const torch::Tensor &packed, int64_t k, int64_t n, int64_t pk, int64_t pn,
            int64_t start_col, int epilogue, int layout, int split_k, cudaStream_t stream) {
    check_cuda_tensors("w4a16 linear", {&out, &in, &packed});
    TORCH_CHECK(packed.scalar_type() == torch::kUInt8 && packed.is_contiguous(), "w4a16 linear: packed must be contiguous uint8");
    TORCH_CHECK(packed.numel() == packed_bytes(pk, pn), "w4a16 linear: packed has ", packed.numel(), " bytes, not those of [", pk, ", ",
                pn, "]");
    TORCH_CHECK(in.stride(-1) == 1 && out.stride(-1) == 1, "w4a16 linear: rows must be contiguous");
    const int64_t m = rows_of(in);
    TORCH_CHECK(rows_of(out) == m, "w4a16 linear: input and output rows differ");
    if (m > 16 && hmb_w4a16_gemm_supports(m, k, n, epilogue)) {
        hmb_check(hmb_w4a16_gemm(static_cast<const uint8_t *>(packed.data_ptr()), pk, pn, in.data_ptr(), ld_of(in), dtype_code(in),
                                 out.data_ptr(), ld_of(out), dtype_code(out), m, k, n, start_col, epilogue, layout, stream),
                  "hmb_w4a16_gemm");
        return;
    }
    const size_t ws_bytes = hmb_w4a16_gemv_workspace(m, k, n, epilogue, split_k);
    torch::Tensor &ws = workspace(in.device(), stream, kWsGemv, ws_bytes);
    hmb_check(hmb_w4a16_gemv(static_cast<const uint8_t *>(packed.data_ptr()), pk, pn, in.data_ptr(), ld_of(in), dtype_code(in),
                             out.data_ptr(), ld_of(out), dtype_code(out), m, k, n, start_col, epilogue, layout, split_k, ws.data_ptr(),
                             static_cast<size_t>(ws.numel()), stream),
              "hmb_w4a16_gemv");
}

cudaStream_t current_stream(const torch::Device &device) { return c10::cuda::getCurrentCUDAStream(device.index()).stream(); }

// Prepared-input bookkeeping of GemmInputReuse, per thread (the class declares no data members):
// the x that residual_norm_bf16 or mark_prepared named last, the object that named it, and the
// number of GEMM calls of each live object that read that x.
struct Prepared {
    const void *x = nullptr;
    int64_t k = 0;
    cudaStream_t stream = nullptr;
    const void *owner = nullptr;
};
thread_local Prepared t_prepared;
thread_local std::map<const void *, int> t_hits;

void note_gemm_input(const void *x, int64_t k, cudaStream_t stream) {
    const Prepared &p = t_prepared;
    if (p.owner && p.x == x && p.k == k && p.stream == stream) ++t_hits[p.owner];
}

}  // namespace

namespace heteromega {

// ---- weight packing ----------------------------------------------------------------------------------

torch::Tensor pack_w4a16(const torch::Tensor &qweight, const torch::Tensor &scales, const torch::Tensor &zeros) {
    TORCH_CHECK(qweight.dim() == 2, "pack_w4a16: qweight must be [K, N]");
    const int64_t K = qweight.size(0), N = qweight.size(1);
    TORCH_CHECK(K % kTileK == 0 && N % kTileN == 0, "pack_w4a16: K must be a multiple of 128 and N of 64, got ", K, "x", N);
    TORCH_CHECK(scales.dim() == 2 && scales.size(0) == K / kTileK && scales.size(1) == N, "pack_w4a16: scales must be [K/128, N]");
    TORCH_CHECK(zeros.dim() == 2 && zeros.size(0) == K / kTileK && zeros.size(1) == N, "pack_w4a16: zeros must be [K/128, N]");
    const torch::Tensor q = qweight.to(torch::kCPU, torch::kUInt8).contiguous();
    const torch::Tensor s = scales.to(torch::kCPU, torch::kBFloat16).contiguous();
    const torch::Tensor z = zeros.to(torch::kCPU, torch::kUInt8).contiguous();
    torch::Tensor out = torch::empty({packed_bytes(K, N)}, torch::TensorOptions().dtype(torch::kUInt8));
    const int rc = hmb_pack_w4a16(q.data_ptr<uint8_t>(), reinterpret_cast<const uint16_t *>(s.data_ptr()), z.data_ptr<uint8_t>(), K, N,
                                  out.data_ptr<uint8_t>());
    TORCH_CHECK(rc != HMB_ERR_VALUE, "pack_w4a16: weights and zeros must lie in 0..15");
    hmb_check(rc, "pack_w4a16");
    return out;
}

FfnSliceWeights FfnSliceWeights::to(const torch::Device &device) const {
    FfnSliceWeights w = *this;
    w.gate_up = gate_up.to(device);
    w.down = down.to(device);
    return w;
}

FfnSliceWeights FfnSliceWeights::prefix(int64_t n) const {
    const int64_t stored = stored_channels();
    TORCH_CHECK(n > 0 && n <= stored && n % kTileK == 0, "FfnSliceWeights::prefix: n must be a multiple of 128 in (0, ", stored,
                "], got ", n);
    TORCH_CHECK(n == stored || layout == GateUpLayout::kInterleaved, "FfnSliceWeights::prefix: a shorter prefix needs GateUpLayout::kInterleaved");
    FfnSliceWeights w = *this;
    w.packed_channels = stored;
    w.end = begin + n;
    return w;
}

namespace {
// Columns of gate and up side by side in `layout` order.
torch::Tensor join_gate_up(const torch::Tensor &g, const torch::Tensor &u, GateUpLayout layout) {
    if (layout == GateUpLayout::kBlocked) return torch::cat({g, u}, 1);
    const int64_t r = g.size(0), n = g.size(1);
    return torch::stack({g.reshape({r, n / kTileN, kTileN}), u.reshape({r, n / kTileN, kTileN})}, 2).reshape({r, 2 * n});
}
}  // namespace

FfnSliceWeights pack_ffn_slice(const FfnLayerQuant &layer, int64_t begin, int64_t end, GateUpLayout layout) {
    TORCH_CHECK(layer.gate_q.dim() == 2, "pack_ffn_slice: gate_q must be [H, I]");
    const int64_t hidden = layer.gate_q.size(0), inter = layer.gate_q.size(1);
    TORCH_CHECK(0 <= begin && begin < end && end <= inter, "pack_ffn_slice: bad channel range [", begin, ", ", end, ")");
    TORCH_CHECK(begin % kTileK == 0 && end % kTileK == 0, "pack_ffn_slice: begin and end must be multiples of 128");
    TORCH_CHECK(layer.down_q.dim() == 2 && layer.down_q.size(0) == inter && layer.down_q.size(1) == hidden, "pack_ffn_slice: down_q must be [I, H]");
    auto cols = [&](const torch::Tensor &t) { return t.narrow(1, begin, end - begin); };
    FfnSliceWeights w;
    w.gate_up = pack_w4a16(join_gate_up(cols(layer.gate_q), cols(layer.up_q), layout), join_gate_up(cols(layer.gate_s), cols(layer.up_s), layout),
                           join_gate_up(cols(layer.gate_z), cols(layer.up_z), layout));
    w.down = pack_w4a16(layer.down_q.narrow(0, begin, end - begin), layer.down_s.narrow(0, begin / kTileK, (end - begin) / kTileK),
                        layer.down_z.narrow(0, begin / kTileK, (end - begin) / kTileK));
    w.begin = begin;
    w.end = end;
    w.hidden = hidden;
    w.layout = layout;
    return w;
}

int64_t packed_tile_index(int64_t c, int64_t r, int64_t tiles_k, int64_t tiles_n) {
    const int64_t v = hmb_packed_tile_index(c, r, tiles_k, tiles_n);
    TORCH_CHECK(v >= 0, "packed_tile_index: tile (", c, ", ", r, ") outside a ", tiles_k, " x ", tiles_n, " matrix");
    return v;
}

FfnSliceWeights slice_packed_ffn(const torch::Tensor &gate, const torch::Tensor &up, const torch::Tensor &down, int64_t hidden,
                                 int64_t inter, int64_t begin, int64_t end, GateUpLayout layout) {
    TORCH_CHECK(hidden % kTileK == 0 && inter % kTileK == 0, "slice_packed_ffn: hidden and inter must be multiples of 128");
    TORCH_CHECK(0 <= begin && begin < end && end <= inter, "slice_packed_ffn: bad channel range [", begin, ", ", end, ")");
    TORCH_CHECK(begin % kTileK == 0 && end % kTileK == 0, "slice_packed_ffn: begin and end must be multiples of 128");
    const int64_t matrix_bytes = packed_bytes(hidden, inter);
    for (const torch::Tensor *t : {&gate, &up, &down}) {
        TORCH_CHECK(t->defined() && t->scalar_type() == torch::kUInt8 && t->is_contiguous() && t->numel() == matrix_bytes,
                    "slice_packed_ffn: expected contiguous uint8 packed matrices of ", matrix_bytes, " bytes");
        TORCH_CHECK(t->device() == gate.device(), "slice_packed_ffn: all matrices must be on one device");
    }
    int64_t gu_count = 0, dn_count = 0;
    hmb_check(hmb_slice_tile_counts(hidden, inter, begin, end, &gu_count, &dn_count), "slice_packed_ffn");
    torch::Tensor gu_map = torch::empty({gu_count}, torch::kInt64), dn_map = torch::empty({dn_count}, torch::kInt64);
    hmb_check(hmb_slice_tile_map(hidden, inter, begin, end, static_cast<int>(layout), gu_map.data_ptr<int64_t>(), dn_map.data_ptr<int64_t>()),
              "slice_packed_ffn");
    const bool whole = begin == 0 && end == inter;
    FfnSliceWeights w;
    w.begin = begin;
    w.end = end;
    w.hidden = hidden;
    w.layout = layout;
    if (gate.is_cuda()) {
        const torch::Device dev = gate.device();
        const cudaStream_t stream = current_stream(dev);
        const int64_t tiles = matrix_bytes / kTileBytes;
        const torch::Tensor gu_idx = gu_map.to(dev), dn_idx = dn_map.to(dev);
        w.gate_up = torch::empty({gu_count * kTileBytes}, gate.options());
        hmb_check(hmb_gather_tiles(gate.data_ptr<uint8_t>(), tiles, up.data_ptr<uint8_t>(), gu_idx.data_ptr<int64_t>(), gu_count,
                                   w.gate_up.data_ptr<uint8_t>(), stream),
                  "slice_packed_ffn");
        if (whole) {
            w.down = down;
        } else {
            w.down = torch::empty({dn_count * kTileBytes}, down.options());
            hmb_check(hmb_gather_tiles(down.data_ptr<uint8_t>(), tiles, nullptr, dn_idx.data_ptr<int64_t>(), dn_count,
                                       w.down.data_ptr<uint8_t>(), stream),
                      "slice_packed_ffn");
        }
        return w;
    }
    const torch::Tensor both = torch::cat({gate.view({-1, kTileBytes}), up.view({-1, kTileBytes})});
    w.gate_up = both.index_select(0, gu_map).view({-1});
    w.down = whole ? down : down.view({-1, kTileBytes}).index_select(0, dn_map).view({-1});
    return w;
}

// ---- kernels -----------------------------------------------------------------------------------------

void silu_mul(const torch::Tensor &gate_up, torch::Tensor &act, hipStream_t stream, GateUpLayout layout) {
    TORCH_CHECK(gate_up.dim() == 2 && act.dim() == 2, "silu_mul: expected 2-D tensors");
    TORCH_CHECK(gate_up.scalar_type() == torch::kBFloat16 && act.scalar_type() == torch::kBFloat16, "silu_mul: expected bf16");
    check_cuda_tensors("silu_mul", {&gate_up, &act});
    const int64_t n = act.size(1);
    TORCH_CHECK(act.size(0) == gate_up.size(0) && gate_up.size(1) == 2 * n, "silu_mul: gate_up must be [M, 2n] and act [M, n]");
    TORCH_CHECK(gate_up.stride(1) == 1 && act.stride(1) == 1, "silu_mul: last dimension must be contiguous");
    hmb_check(hmb_silu_mul(gate_up.data_ptr(), gate_up.stride(0), act.data_ptr(), act.stride(0), act.size(0), n, static_cast<int>(layout), stream),
              "silu_mul");
}

void gemv_w4a16(torch::Tensor &out, const torch::Tensor &x, const torch::Tensor &packed, int64_t k, int64_t n, int64_t packed_k,
                int64_t packed_n, int split_k, hipStream_t stream) {
    TORCH_CHECK(k > 0 && n > 0 && k % kTileK == 0 && n % kTileN == 0, "gemv_w4a16: k must be a multiple of 128 and n of 64");
    TORCH_CHECK(k <= packed_k && n <= packed_n && packed_k % kTileK == 0 && packed_n % kTileN == 0, "gemv_w4a16: packed matrix [",
                packed_k, ", ", packed_n, "] does not contain [", k, ", ", n, "]");
    TORCH_CHECK(x.numel() == k && x.is_contiguous() && x.scalar_type() == torch::kBFloat16, "gemv_w4a16: x must be contiguous bf16 with ", k,
                " elements");
    TORCH_CHECK(out.numel() == n && out.is_contiguous() && out.scalar_type() == torch::kBFloat16, "gemv_w4a16: out must be contiguous bf16 with ",
                n, " elements");
    torch::Tensor o = out.view({1, n});
    linear(o, x.view({1, k}), packed, k, n, packed_k, packed_n, 0, HMB_EPI_STORE, 0, split_k, stream);
}

bool gemm_w4a16_supports(int64_t m, int64_t k, int64_t n) { return m > 0 && k > 0 && n > 0 && k % kTileK == 0 && n % kTileN == 0; }

void gemm_w4a16(torch::Tensor &out, const torch::Tensor &x, const torch::Tensor &packed, int64_t k, int64_t n, int64_t packed_k,
                int64_t packed_n, hipStream_t stream) {
    TORCH_CHECK(gemm_w4a16_supports(rows_of(x), k, n), "gemm_w4a16: unsupported shape");
    TORCH_CHECK(k <= packed_k && n <= packed_n, "gemm_w4a16: packed matrix [", packed_k, ", ", packed_n, "] does not contain [", k, ", ", n, "]");
    note_gemm_input(x.data_ptr(), k, stream);
    linear(out, x, packed, k, n, packed_k, packed_n, 0, HMB_EPI_STORE, 0, 0, stream);
}

torch::Tensor gemm_uncached_weights(const torch::Tensor &packed) {
    // The B200 GEMMs read the packed weights where they are: no second copy is made.
    return packed;
}

bool gemm_w4a16_ffn_supports(int64_t m, int64_t h, int64_t n) { return m > 0 && h % kTileK == 0 && n > 0 && n % kTileK == 0; }

void gemm_w4a16_ffn(torch::Tensor &y, const torch::Tensor &x, const torch::Tensor &gate_up, const torch::Tensor &down, int64_t h, int64_t n,
                    int64_t stored, hipStream_t stream) {
    TORCH_CHECK(gemm_w4a16_ffn_supports(rows_of(x), h, n) && n <= stored, "gemm_w4a16_ffn: unsupported shape");
    FfnSliceWeights w;
    w.gate_up = gate_up;
    w.down = down;
    w.begin = 0;
    w.end = n;
    w.hidden = h;
    w.layout = GateUpLayout::kInterleaved;
    w.packed_channels = stored;
    GpuFfnBuffers unused;
    gpu_ffn_slice_forward(w, x, unused, y, stream);
}

GemmInputReuse::GemmInputReuse() { t_hits[this] = 0; }

GemmInputReuse::~GemmInputReuse() {
    t_hits.erase(this);
    if (t_prepared.owner == this) t_prepared = Prepared{};
}

void GemmInputReuse::mark_prepared(const void *x, int64_t k, hipStream_t stream) { t_prepared = Prepared{x, k, stream, this}; }

int GemmInputReuse::hits() const {
    const auto it = t_hits.find(this);
    return it == t_hits.end() ? 0 : it->second;
}

void gemm_input_buffers(int64_t, int64_t, hipStream_t, float **sums, uint16_t **tiles) {
    // The B200 GEMMs read x as it is and form their own row sums: there is no prepared-input buffer.
    if (sums) *sums = nullptr;
    if (tiles) *tiles = nullptr;
}

bool residual_norm_supports(int64_t m, int64_t h) { return m > 0 && h > 0 && h % 8 == 0 && h <= 16384; }

void residual_norm_bf16(uint16_t *x, const uint16_t *a, const uint16_t *b, const uint16_t *weight, uint16_t *normed, const void *gemm_x,
                        GemmInputReuse &gemm_input, int64_t m, int64_t h, int64_t x_stride, int64_t a_stride, int64_t b_stride,
                        int64_t normed_stride, float eps, hipStream_t stream) {
    TORCH_CHECK(residual_norm_supports(m, h), "residual_norm_bf16: unsupported shape ", m, "x", h);
    TORCH_CHECK(b == nullptr || a != nullptr, "residual_norm_bf16: b needs a");
    uint16_t *dst = normed;
    int64_t dst_stride = normed_stride;
    if (dst == nullptr && gemm_x != nullptr) {
        // The next GEMM reads x = gemm_x (rows of h values): the normed rows go there.
        dst = static_cast<uint16_t *>(const_cast<void *>(gemm_x));
        dst_stride = h;
    }
    hmb_check(hmb_residual_norm(x, x_stride, a, a_stride, b, b_stride, weight, dst, dst_stride, m, h, eps, stream), "residual_norm_bf16");
    if (gemm_x != nullptr) gemm_input.mark_prepared(gemm_x, h, stream);
}

void residual_add2(torch::Tensor &x, const torch::Tensor &y_g, const torch::Tensor &y_n, hipStream_t stream) {
    check_cuda_tensors("residual_add2", {&x, &y_g, &y_n});
    TORCH_CHECK(x.scalar_type() == torch::kBFloat16, "residual_add2: x must be bf16");
    TORCH_CHECK(x.dim() >= 1 && x.stride(-1) == 1 && y_g.stride(-1) == 1 && y_n.stride(-1) == 1, "residual_add2: rows must be contiguous");
    const int64_t cols = x.size(-1), m = x.numel() / cols;
    TORCH_CHECK(y_g.numel() == x.numel() && y_n.numel() == x.numel(), "residual_add2: shapes differ");
    TORCH_CHECK(x.is_contiguous() && y_g.is_contiguous() && y_n.is_contiguous(), "residual_add2: tensors must be contiguous");
    hmb_check(hmb_residual_add2(x.data_ptr(), cols, y_g.data_ptr(), cols, dtype_code(y_g), y_n.data_ptr(), cols, dtype_code(y_n), m, cols, stream),
              "residual_add2");
}

void residual_add2_cpu(torch::Tensor &x, const torch::Tensor &y_g, const torch::Tensor &y_n) {
    // x += y_g + y_n on host tensors: the partials first, in fp32, then one bf16 rounding.
    TORCH_CHECK(!x.is_cuda() && !y_g.is_cuda() && !y_n.is_cuda(), "residual_add2_cpu: expected CPU tensors");
    TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.numel() == y_g.numel() && x.numel() == y_n.numel(), "residual_add2_cpu: shapes differ");
    const torch::Tensor sum = y_g.to(torch::kFloat).reshape(x.sizes()) + y_n.to(torch::kFloat).reshape(x.sizes());
    x.copy_((x.to(torch::kFloat) + sum).to(torch::kBFloat16));
}

// ---- the GPU slice ---------------------------------------------------------------------------------------

GpuFfnBuffers GpuFfnBuffers::allocate(int64_t max_m, int64_t channels, int64_t hidden, const torch::Device &device) {
    // The activation lives in the library's workspace and gate/up never reaches memory; the buffers are
    // kept for callers that pass them around, sized for the largest call.
    const auto opt = torch::TensorOptions().dtype(torch::kBFloat16).device(device);
    return {torch::empty({0, 2 * channels}, opt), torch::empty({max_m, channels}, opt), torch::empty({max_m, hidden}, opt)};
}

void gpu_ffn_slice_forward(const FfnSliceWeights &w, const torch::Tensor &x_norm, GpuFfnBuffers &, torch::Tensor &y, hipStream_t stream) {
    const int64_t n = w.channels(), stored = w.stored_channels(), h = w.hidden;
    TORCH_CHECK(n == stored || w.layout == GateUpLayout::kInterleaved,
                "gpu_ffn_slice_forward: a prefix of the packed channels needs GateUpLayout::kInterleaved");
    TORCH_CHECK(x_norm.dim() == 2 && x_norm.size(1) == h && x_norm.stride(1) == 1, "gpu_ffn_slice_forward: x_norm must be contiguous [M, H]");
    const int64_t m = x_norm.size(0);
    TORCH_CHECK(y.dim() == 2 && y.size(0) == m && y.size(1) == h && y.stride(1) == 1, "gpu_ffn_slice_forward: y must be [M, H]");
    check_cuda_tensors("gpu_ffn_slice_forward", {&x_norm, &y, &w.gate_up, &w.down});
    TORCH_CHECK(w.gate_up.numel() == packed_bytes(h, 2 * stored) && w.down.numel() == packed_bytes(stored, h),
                "gpu_ffn_slice_forward: packed sizes do not match H = ", h, ", ", stored, " channels");
    note_gemm_input(x_norm.data_ptr(), h, stream);
    const size_t ws_bytes = hmb_w4a16_ffn_workspace(m, h, n);
    torch::Tensor &ws = workspace(x_norm.device(), stream, kWsFfn, ws_bytes);
    hmb_check(hmb_w4a16_ffn(w.gate_up.data_ptr<uint8_t>(), w.down.data_ptr<uint8_t>(), h, n, stored, static_cast<int>(w.layout),
                            x_norm.data_ptr(), x_norm.stride(0), dtype_code(x_norm), y.data_ptr(), y.stride(0), dtype_code(y), m,
                            ws.data_ptr(), static_cast<size_t>(ws.numel()), stream),
              "gpu_ffn_slice_forward");
}

GemmKernel configured_gemm_kernel() {
    static const GemmKernel kernel = [] {
        const char *v = std::getenv("HETEROMEGA_GEMM");
        return v != nullptr && std::string(v) == "fast" ? GemmKernel::kHeteroMega : GemmKernel::kHeteroMosaic;
    }();
    return kernel;
}

void packed_linear(torch::Tensor &out, const torch::Tensor &in, const torch::Tensor &packed, int64_t k, int64_t n, hipStream_t stream,
                   const LinearOptions &opt) {
    const int64_t pk = opt.packed_k > 0 ? opt.packed_k : k;
    const int64_t pn = opt.packed_n > 0 ? opt.packed_n : n;
    TORCH_CHECK(in.dim() == 2 && in.size(1) == k && in.stride(1) == 1, "packed_linear: input must be contiguous [M, ", k, "]");
    const int64_t m = in.size(0);
    TORCH_CHECK(m > 0, "packed_linear: M must be > 0");
    TORCH_CHECK(k % kTileK == 0 && n % kTileN == 0, "packed_linear: k must be a multiple of 128 and n of 64");
    const int64_t out_n = opt.fuse_activation ? n / 2 : n;
    TORCH_CHECK(!opt.fuse_activation || n % (2 * kTileN) == 0, "packed_linear: fused activation needs a gate/up width that is a multiple of 128");
    TORCH_CHECK(out.dim() == 2 && out.size(0) == m && out.size(1) == out_n && out.stride(1) == 1, "packed_linear: output must be contiguous [M, ",
                out_n, "]");
    TORCH_CHECK(in.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kBFloat16, "packed_linear: expected bf16");
    TORCH_CHECK(k <= pk && n <= pn && pk % kTileK == 0 && pn % kTileN == 0, "packed_linear: packed matrix [", pk, ", ", pn, "] does not contain [",
                k, ", ", n, "]");
    TORCH_CHECK(packed.numel() == packed_bytes(pk, pn), "packed_linear: packed size does not match ", pk, "x", pn);
    TORCH_CHECK(packed.device() == in.device() && out.device() == in.device(), "packed_linear: all tensors must be on one device");
    note_gemm_input(in.data_ptr(), k, stream);
    // fuse_activation: the reference's gate/up matrices are interleaved (the GpuFfnModel and
    // slice_packed_ffn default to it for the fused path).
    linear(out, in, packed, k, n, pk, pn, 0, opt.fuse_activation ? HMB_EPI_SWIGLU : HMB_EPI_STORE, HMB_GATE_UP_INTERLEAVED, opt.gemv_split_k,
           stream);
}

// ---- model integration ------------------------------------------------------------------------------------

void GpuFfnModel::add_layer(const torch::Tensor &gate, const torch::Tensor &up, const torch::Tensor &down, int64_t hidden, int64_t inter) {
    TORCH_CHECK(layers_.empty() || (layers_.front().hidden == hidden && layers_.front().stored_channels() == inter),
                "GpuFfnModel::add_layer: all layers must have the same shape");
    layers_.push_back(slice_packed_ffn(gate, up, down, hidden, inter, 0, inter, GateUpLayout::kInterleaved));
    if (s_prefill_ == 0) s_prefill_ = s_decode_ = inter;
}

void GpuFfnModel::set_split(int64_t s_prefill, int64_t s_decode) {
    TORCH_CHECK(!layers_.empty(), "GpuFfnModel::set_split: add the layers first");
    const int64_t inter = layers_.front().stored_channels();
    for (int64_t s : {s_prefill, s_decode})
        TORCH_CHECK(s > 0 && s <= inter && s % kTileK == 0, "GpuFfnModel::set_split: channels must be a multiple of 128 in (0, ", inter, "], got ", s);
    s_prefill_ = s_prefill;
    s_decode_ = s_decode;
}

void GpuFfnModel::forward(int64_t layer, const torch::Tensor &x_norm, torch::Tensor &y, hipStream_t stream) {
    TORCH_CHECK(0 <= layer && layer < layers(), "GpuFfnModel::forward: no layer ", layer);
    const FfnSliceWeights &all = layers_[layer];
    GpuFfnBuffers *buf = nullptr;
    {
        std::lock_guard<std::mutex> lock(mutex_);
        buf = &buffers_[stream];  // kept per stream, as the reference keeps its scratch
    }
    gpu_ffn_slice_forward(all.prefix(channels(x_norm.size(0))), x_norm, *buf, y, stream);
}

}  // namespace heteromega

// ---- HeteroMosaic's kernel API (include/hipkernels/w4a16_gemm_packed.hpp) ------------------------------------

namespace hipkernels {

void w4a16_gemm_fused_packed(torch::Tensor &output, const torch::Tensor &input, const torch::Tensor &packed_params, int64_t in_features,
                             int64_t out_features, hipStream_t stream) {
    w4a16_gemm_fused_packed_tiles(output, input, packed_params, in_features, out_features, in_features / heteromega::kTileK,
                                  out_features / heteromega::kTileN, stream, false);
}

void w4a16_gemm_fused_packed_tiles(torch::Tensor &output, const torch::Tensor &input, const torch::Tensor &packed_params, int64_t in_features,
                                   int64_t out_features, int64_t packed_tiles_k, int64_t packed_tiles_n, hipStream_t stream, bool fuse_activation) {
    // [batch, seq, features] or [rows, features]: rows are flattened.
    TORCH_CHECK(input.size(-1) == in_features && input.is_contiguous(), "w4a16_gemm_fused_packed: input must be contiguous [..., ", in_features, "]");
    const int64_t out_n = fuse_activation ? out_features / 2 : out_features;
    TORCH_CHECK(output.size(-1) == out_n && output.is_contiguous(), "w4a16_gemm_fused_packed: output must be contiguous [..., ", out_n, "]");
    const torch::Tensor in2 = input.view({-1, in_features});
    torch::Tensor out2 = output.view({-1, out_n});
    linear(out2, in2, packed_params, in_features, out_features, packed_tiles_k * heteromega::kTileK, packed_tiles_n * heteromega::kTileN, 0,
           fuse_activation ? HMB_EPI_SWIGLU : HMB_EPI_STORE, HMB_GATE_UP_INTERLEAVED, 0, stream);
}

void w4a16_gemv_fused_packed(torch::Tensor &output, const torch::Tensor &input, const torch::Tensor &packed_params, int64_t in_features,
                             int64_t out_features, int64_t total_out_features, int64_t start_col, hipStream_t stream) {
    // Columns [start_col, start_col + out_features) of a packed [in_features, total_out_features] matrix,
    // for row 0 of the input (the reference's GEMV reads one token).
    const int64_t total = total_out_features > 0 ? total_out_features : out_features;
    TORCH_CHECK(input.numel() >= in_features && input.is_contiguous(), "w4a16_gemv_fused_packed: input must hold ", in_features, " contiguous values");
    TORCH_CHECK(output.numel() >= out_features && output.is_contiguous(), "w4a16_gemv_fused_packed: output must hold ", out_features, " values");
    TORCH_CHECK(start_col >= 0 && start_col + out_features <= total, "w4a16_gemv_fused_packed: columns outside the packed matrix");
    const torch::Tensor x = input.view({-1}).narrow(0, 0, in_features).view({1, in_features});
    torch::Tensor y = output.view({-1}).narrow(0, 0, out_features).view({1, out_features});
    linear(y, x, packed_params, in_features, out_features, in_features, total, start_col, HMB_EPI_STORE, 0, 0, stream);
}

void w4a16_gemm_wmma_packed(torch::Tensor &output, const torch::Tensor &input, const torch::Tensor &packed_params, int64_t in_features,
                            int64_t out_features) {
    w4a16_gemm_fused_packed(output, input, packed_params, in_features, out_features, current_stream(input.device()));
}

bool is_hip_available() { return torch::cuda::is_available(); }

void hip_synchronize() { torch::cuda::synchronize(); }

}  // namespace hipkernels
