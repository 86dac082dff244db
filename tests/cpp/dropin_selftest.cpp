// TEST INFRASTRUCTURE: a C++ caller of the reference's FFN interface (heteromega/gpu_ffn.hpp and
// hipkernels/w4a16_gemm_packed.hpp, compiled unchanged) linked to libhmb_dropin.so, run on a GPU by
// tests/test_cpp_dropin_gpu.py. It calls the API the way the reference's code does:
//   * the model loop: GpuFfnModel::add_layer for every layer, set_split(s_prefill, s_decode), then
//     forward(layer, x_norm, y, stream) for a decode token and a prefill chunk
//     (src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2852-2865, 2377-2382);
//   * the GEMV/GEMM dispatch: hipkernels::w4a16_gemv_fused_packed with total_out_features and
//     start_col, w4a16_gemm_fused_packed_tiles with and without fuse_activation
//     (include/unified_llm_w4a16_hetero/hetero_compute.hpp:16-39);
//   * heteromega::gemm_w4a16_ffn, packed_linear, silu_mul, residual_add2, residual_norm_bf16 with a
//     GemmInputReuse, pack_ffn_slice against slice_packed_ffn.
// Each result is compared with a torch fp32 reference of the packed format's definition: weights
// dequantised by hmb_w4a16_dequant ((q - z) * s, exact), fp32 matmuls, gate and up rounded to bf16,
// SiLU * up rounded once (the reference GEMM's arithmetic apart from its weight rounding). The
// program prints one line per check and exits 1 if a check exceeds max |err| / max |ref| <= 1e-2.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <heteromega/gpu_ffn.hpp>
#include <hipkernels/w4a16_gemm_packed.hpp>
#include <torch/cuda.h>

#include <cstdio>
#include <cstring>

#include "hmb.h"

namespace {

int g_failures = 0;

void report(const char *what, const torch::Tensor &got, const torch::Tensor &ref, double tol = 1e-2) {
    const torch::Tensor g = got.to(torch::kCPU, torch::kDouble), r = ref.to(torch::kCPU, torch::kDouble);
    const double max_ref = r.abs().max().item<double>();
    const double max_rel = (g - r).abs().max().item<double>() / (max_ref > 0 ? max_ref : 1.0);
    const double rel_l2 = (g - r).norm().item<double>() / (r.norm().item<double>() + 1e-30);
    const bool ok = max_rel <= tol && rel_l2 <= tol && std::isfinite(max_rel);
    std::printf("%-58s max_rel %.3e rel_l2 %.3e %s\n", what, max_rel, rel_l2, ok ? "ok" : "FAIL");
    if (!ok) ++g_failures;
}

void expect(const char *what, bool ok) {
    std::printf("%-58s %s\n", what, ok ? "ok" : "FAIL");
    if (!ok) ++g_failures;
}

struct Quant {
    torch::Tensor q, s, z;  // [K, N] uint8, [K/128, N] bf16, [K/128, N] int8 (CPU)
};

Quant random_quant(int64_t k, int64_t n) {
    Quant w;
    w.q = torch::randint(0, 16, {k, n}, torch::kUInt8);
    w.s = (torch::rand({k / 128, n}) * 0.018 + 0.002).to(torch::kBFloat16);
    w.z = torch::randint(0, 16, {k / 128, n}, torch::kInt8);
    return w;
}

// fp32 [k, n] = (q - z) * s of the leading [k, n] block of a packed [pk, pn] matrix on the device.
torch::Tensor dequant(const torch::Tensor &packed, int64_t pk, int64_t pn, int64_t k, int64_t n, cudaStream_t stream) {
    torch::Tensor out = torch::empty({k, n}, packed.options().dtype(torch::kFloat));
    const int rc = hmb_w4a16_dequant(packed.data_ptr<uint8_t>(), pk, pn, k, n, out.data_ptr<float>(), n, stream);
    TORCH_CHECK(rc == HMB_OK, "hmb_w4a16_dequant failed: ", rc);
    return out;
}

torch::Tensor bf(const torch::Tensor &t) { return t.to(torch::kBFloat16).to(torch::kFloat); }

// The FFN of channels [0, s) of whole gate [H, I], up [H, I], down [I, H] (fp32 weights) for x.
torch::Tensor ffn_ref(const torch::Tensor &x, const torch::Tensor &wg, const torch::Tensor &wu, const torch::Tensor &wd, int64_t s) {
    const torch::Tensor xf = x.to(torch::kFloat);
    const torch::Tensor g = bf(xf.matmul(wg.narrow(1, 0, s))), u = bf(xf.matmul(wu.narrow(1, 0, s)));
    const torch::Tensor act = bf(g / (1 + torch::exp(-g)) * u);
    return act.matmul(wd.narrow(0, 0, s));
}

}  // namespace

int main() {
    if (!torch::cuda::is_available()) {
        std::printf("no CUDA device\n");
        return 2;
    }
    at::globalContext().setAllowTF32CuBLAS(false);
    torch::manual_seed(5);
    const torch::Device dev(torch::kCUDA, 0);
    const auto bf16 = torch::TensorOptions().dtype(torch::kBFloat16).device(dev);
    c10::cuda::CUDAStream side = c10::cuda::getStreamFromPool(false, 0);
    c10::cuda::CUDAStreamGuard guard(side);
    const cudaStream_t stream = side.stream();

    // Llama-3.2-1B FFN shape, two layers.
    const int64_t H = 2048, I = 8192, L = 2;
    heteromega::GpuFfnModel model;
    std::vector<std::array<torch::Tensor, 3>> dense;  // fp32 gate, up, down per layer
    std::vector<std::array<torch::Tensor, 3>> packed;
    for (int64_t l = 0; l < L; ++l) {
        const Quant g = random_quant(H, I), u = random_quant(H, I), d = random_quant(I, H);
        const torch::Tensor pg = heteromega::pack_w4a16(g.q, g.s, g.z).to(dev);
        const torch::Tensor pu = heteromega::pack_w4a16(u.q, u.s, u.z).to(dev);
        const torch::Tensor pd = heteromega::pack_w4a16(d.q, d.s, d.z).to(dev);
        model.add_layer(pg, pu, pd, H, I);
        packed.push_back({pg, pu, pd});
        dense.push_back({dequant(pg, H, I, H, I, stream), dequant(pu, H, I, H, I, stream), dequant(pd, I, H, I, H, stream)});
    }
    expect("GpuFfnModel::add_layer x2", model.layers() == L);
    const int64_t s_prefill = 6144, s_decode = 4096;
    model.set_split(s_prefill, s_decode);
    expect("GpuFfnModel::set_split channels(1), channels(300)", model.channels(1) == s_decode && model.channels(300) == s_prefill);

    for (int64_t m : {1, 300}) {
        for (int64_t l = 0; l < L; ++l) {
            const torch::Tensor x = torch::randn({m, H}, bf16);
            torch::Tensor y = torch::empty({m, H}, bf16);
            model.forward(l, x, y, stream);
            side.synchronize();
            const torch::Tensor ref = ffn_ref(x, dense[l][0], dense[l][1], dense[l][2], model.channels(m));
            char what[96];
            std::snprintf(what, sizeof what, "GpuFfnModel::forward layer %ld M=%ld (%ld channels)", l, m, model.channels(m));
            report(what, y, ref);
        }
    }

    // HeteroMosaic's GEMV: a column window of the whole packed gate matrix, one token.
    {
        const torch::Tensor x = torch::randn({1, H}, bf16);
        torch::Tensor y = torch::empty({1, 1024}, bf16);
        hipkernels::w4a16_gemv_fused_packed(y, x, packed[0][0], H, 1024, I, 2048, stream);
        side.synchronize();
        report("hipkernels::w4a16_gemv_fused_packed cols 2048..3071", y, x.to(torch::kFloat).matmul(dense[0][0].narrow(1, 2048, 1024)));
    }
    // HeteroMosaic's GEMM over the interleaved gate_up slice, plain and with fuse_activation.
    {
        const heteromega::FfnSliceWeights w =
            heteromega::slice_packed_ffn(packed[1][0], packed[1][1], packed[1][2], H, I, 0, I, heteromega::GateUpLayout::kInterleaved);
        const torch::Tensor x = torch::randn({2, 100, H}, bf16);
        torch::Tensor act = torch::empty({2, 100, I}, bf16);
        hipkernels::w4a16_gemm_fused_packed_tiles(act, x, w.gate_up, H, 2 * I, H / 128, 2 * I / 64, stream, true);
        torch::Tensor down_out = torch::empty({2, 100, H}, bf16);
        hipkernels::w4a16_gemm_fused_packed(down_out, act, w.down, I, H, stream);
        side.synchronize();
        const torch::Tensor xf = x.view({200, H}).to(torch::kFloat);
        const torch::Tensor g = bf(xf.matmul(dense[1][0])), u = bf(xf.matmul(dense[1][1]));
        report("hipkernels::w4a16_gemm_fused_packed_tiles fuse_activation", act.view({200, I}), g / (1 + torch::exp(-g)) * u);
        report("hipkernels::w4a16_gemm_fused_packed (down)", down_out.view({200, H}), act.view({200, I}).to(torch::kFloat).matmul(dense[1][2]));

        // heteromega::gemm_w4a16_ffn on a channel prefix of the same slice.
        torch::Tensor y = torch::empty({200, H}, bf16);
        heteromega::gemm_w4a16_ffn(y, x.view({200, H}), w.gate_up, w.down, H, 2048, I, stream);
        side.synchronize();
        report("heteromega::gemm_w4a16_ffn 2048 of 8192 channels", y, ffn_ref(x.view({200, H}), dense[1][0], dense[1][1], dense[1][2], 2048));

        // packed_linear: GEMV for one row, GEMM for 64, and the fused activation.
        heteromega::LinearOptions opt;
        for (int64_t m : {1, 64}) {
            const torch::Tensor xi = torch::randn({m, I}, bf16);
            torch::Tensor out = torch::empty({m, H}, bf16);
            heteromega::packed_linear(out, xi, w.down, I, H, stream, opt);
            side.synchronize();
            char what[96];
            std::snprintf(what, sizeof what, "heteromega::packed_linear down M=%ld", m);
            report(what, out, xi.to(torch::kFloat).matmul(dense[1][2]));
        }
    }
    // silu_mul and residual_add2.
    {
        const torch::Tensor gu = torch::randn({37, 2 * 512}, bf16) * 3;
        torch::Tensor act = torch::empty({37, 512}, bf16);
        heteromega::silu_mul(gu, act, stream, heteromega::GateUpLayout::kBlocked);
        torch::Tensor x = torch::randn({37, H}, bf16);
        const torch::Tensor x0 = x.clone(), yg = torch::randn({37, H}, bf16), yn = torch::randn({37, H}, bf16.dtype(torch::kFloat));
        heteromega::residual_add2(x, yg, yn, stream);
        side.synchronize();
        const torch::Tensor g = gu.narrow(1, 0, 512).to(torch::kFloat), u = gu.narrow(1, 512, 512).to(torch::kFloat);
        report("heteromega::silu_mul", act, g / (1 + torch::exp(-g)) * u, 1e-2);
        expect("heteromega::residual_add2 bit for bit", torch::equal(x, (x0.to(torch::kFloat) + (yg.to(torch::kFloat) + yn)).to(torch::kBFloat16)));
    }
    // residual_norm_bf16 feeding the next GEMM through GemmInputReuse, as the model's boundary does.
    {
        const int64_t m = 64;
        torch::Tensor x = torch::randn({m, H}, bf16);
        const torch::Tensor x0 = x.clone(), a = torch::randn({m, H}, bf16), w = (torch::randn({H}) * 0.2 + 1).to(bf16);
        torch::Tensor normed = torch::empty({m, H}, bf16);
        heteromega::GemmInputReuse reuse;
        heteromega::residual_norm_bf16(reinterpret_cast<uint16_t *>(x.data_ptr()), reinterpret_cast<const uint16_t *>(a.data_ptr()), nullptr,
                                       reinterpret_cast<const uint16_t *>(w.data_ptr()), nullptr, normed.data_ptr(), reuse, m, H, H, H, 0, H,
                                       1e-5f, stream);
        torch::Tensor out = torch::empty({m, I}, bf16);
        heteromega::gemm_w4a16(out, normed, packed[0][0], H, I, H, I, stream);
        side.synchronize();
        const torch::Tensor xs = (x0.to(torch::kFloat) + a.to(torch::kFloat)).to(torch::kBFloat16).to(torch::kFloat);
        const torch::Tensor nr = bf(xs * torch::rsqrt(xs.pow(2).mean(-1, true) + 1e-5) * w.to(torch::kFloat));
        expect("heteromega::residual_norm_bf16 residual bit for bit", torch::equal(x, xs.to(torch::kBFloat16)));
        report("heteromega::residual_norm_bf16 normed rows (gemm_x)", normed, nr, 8e-3);
        expect("GemmInputReuse::hits() after one GEMM on gemm_x", reuse.hits() == 1);
        report("heteromega::gemm_w4a16 on the prepared input", out, normed.to(torch::kFloat).matmul(dense[0][0]));
    }
    // pack_ffn_slice (from AWQ-order tensors) gives the bytes of slice_packed_ffn (from packed ones).
    {
        const Quant g = random_quant(512, 1024), u = random_quant(512, 1024), d = random_quant(1024, 512);
        heteromega::FfnLayerQuant layer{g.q, g.s, g.z, u.q, u.s, u.z, d.q, d.s, d.z};
        const torch::Tensor pg = heteromega::pack_w4a16(g.q, g.s, g.z), pu = heteromega::pack_w4a16(u.q, u.s, u.z),
                            pd = heteromega::pack_w4a16(d.q, d.s, d.z);
        bool same = true;
        for (auto layout : {heteromega::GateUpLayout::kBlocked, heteromega::GateUpLayout::kInterleaved}) {
            const auto a = heteromega::pack_ffn_slice(layer, 256, 768, layout);
            const auto b = heteromega::slice_packed_ffn(pg, pu, pd, 512, 1024, 256, 768, layout);
            const auto c = heteromega::slice_packed_ffn(pg.to(dev), pu.to(dev), pd.to(dev), 512, 1024, 256, 768, layout);
            same = same && torch::equal(a.gate_up, b.gate_up) && torch::equal(a.down, b.down) && torch::equal(a.gate_up, c.gate_up.cpu()) &&
                   torch::equal(a.down, c.down.cpu());
        }
        expect("pack_ffn_slice == slice_packed_ffn (host and device)", same);
        bool threw = false;
        try {
            model.set_split(100, 128);
        } catch (const c10::Error &) {
            threw = true;
        }
        expect("GpuFfnModel::set_split rejects 100 channels (TORCH_CHECK)", threw);
    }
    int status = 0;
    expect("hmb_device_status clear", hmb_device_status(&status, stream) == HMB_OK && status == HMB_OK);
    std::printf("%s: %d failure(s)\n", g_failures ? "FAILED" : "PASSED", g_failures);
    return g_failures ? 1 : 0;
}
