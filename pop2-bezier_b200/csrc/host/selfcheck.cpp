// On-device self-checks: the one run before int8 caches are created, and the
// one that gates the optional fused float-KV decode kernels.
//
// Restates the reference's preparation check, app/src/model/int8_kv_ops.rs:57-103:
// the same closed-form fixtures, the same host loops, the same tolerances and
// the same failure messages (which app/src/inference.rs:84-92 classifies as a
// safe fallback to floating KV).  The device path exercised is the product
// path: pp_b200_quantize, pp_b200_dequantize and pp_b200_decode_attention.
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "internal.h"

namespace {

struct DevBuf {
    void* p = nullptr;
    cudaError_t alloc(size_t n) { return cudaMalloc(&p, n ? n : 1); }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

#define PP_TRY_CUDA(expr)                                                                              \
    do {                                                                                               \
        cudaError_t e_ = (expr);                                                                       \
        if (e_ != cudaSuccess) {                                                                       \
            std::string m = std::string("EXECUTION_UNCERTAIN: KV INT8 preparation: ") + #expr + ": " + \
                            cudaGetErrorName(e_);                                                      \
            if (e_ == cudaErrorMemoryAllocation) m = std::string("KV INT8 preparation: ") + cudaGetErrorName(e_); \
            return pp::fail_msg(e_ == cudaErrorMemoryAllocation ? PP_STATUS_PRECONDITION : PP_STATUS_UNCERTAIN, m.c_str()); \
        }                                                                                              \
    } while (0)

#define PP_TRY(expr)               \
    do {                           \
        int32_t s_ = (expr);       \
        if (s_ != PP_STATUS_OK) return s_; \
    } while (0)

// Host loop of int8_kv_ops.rs:69-73 / :95-99 for one row: history from the
// bf16-rounded dequantized arena, scratch token last.
void expected_row(const float* q, const float* kc, const float* vc, const float* sk, const float* sv, uint32_t len,
                  float* out) {
    std::vector<float> scores(len + 1);
    float mx = -INFINITY;
    for (uint32_t t = 0; t <= len; ++t) {
        float acc = 0.f;
        for (int d = 0; d < 64; ++d) acc += q[d] * (t == len ? sk[d] : kc[t * 64 + d]);
        scores[t] = acc * 0.125f;
        mx = std::fmax(mx, scores[t]);
    }
    float z = 0.f;
    for (auto& s : scores) {
        s = std::exp(s - mx);
        z += s;
    }
    for (int d = 0; d < 64; ++d) {
        float acc = 0.f;
        for (uint32_t t = 0; t <= len; ++t) acc += scores[t] * (t == len ? sv[d] : vc[t * 64 + d]);
        out[d] = acc / z;
    }
}

int32_t run_attention(const PpKvArena& arena, uint32_t split, const float* q, const float* sk, const float* sv,
                      const uint32_t* past, float* out) {
    PpAttnParams p{};
    p.struct_size = sizeof p;
    p.split_tokens = split;
    p.q_dtype = PP_DTYPE_F32;
    p.out_dtype = PP_DTYPE_F32;
    const size_t ws_bytes = pp_b200_attention_workspace_size(&arena, &p);
    DevBuf ws;
    PP_TRY_CUDA(ws.alloc(ws_bytes));
    PP_TRY(pp_b200_decode_attention(&arena, &p, q, sk, sv, past, out, ws.p, ws_bytes, nullptr, nullptr));
    PP_TRY_CUDA(cudaDeviceSynchronize());
    return PP_STATUS_OK;
}

int32_t selfcheck() {
    // ---- fixture 1: 2 heads x 3 tokens, quantize round trip, then attention.
    std::vector<float> data(384);
    for (int i = 0; i < 384; ++i) data[i] = std::sin((float)i * 0.17f) * 2.f;
    DevBuf dx, dk, ds, drest;
    PP_TRY_CUDA(dx.alloc(384 * 4));
    PP_TRY_CUDA(dk.alloc(384));
    PP_TRY_CUDA(ds.alloc(6 * 4));
    PP_TRY_CUDA(drest.alloc(384 * 4));
    PP_TRY_CUDA(cudaMemcpy(dx.p, data.data(), 384 * 4, cudaMemcpyHostToDevice));
    PP_TRY(pp_b200_quantize(dx.p, PP_DTYPE_F32, 6, 64, (uint8_t*)dk.p, (float*)ds.p, nullptr, nullptr));
    PP_TRY(pp_b200_dequantize((const uint8_t*)dk.p, (const float*)ds.p, 6, 64, 0, PP_DTYPE_F32, drest.p, nullptr));
    std::vector<float> restored(384);
    PP_TRY_CUDA(cudaMemcpy(restored.data(), drest.p, 384 * 4, cudaMemcpyDeviceToHost));
    for (int i = 0; i < 384; ++i)
        if (!std::isfinite(restored[i]) || std::fabs(restored[i] - data[i]) >= 0.009f)
            return pp::fail_msg(PP_STATUS_PRECONDITION, "KV INT8 quantization self-check failed");

    std::vector<float> qdata(128), scratch(128);
    for (int i = 0; i < 128; ++i) {
        qdata[i] = std::cos((float)i * 0.07f);
        scratch[i] = std::sin((float)i * 0.09f);
    }
    const uint32_t past1[2] = {2, 1};
    DevBuf dq, dsk, dpast, dout;
    PP_TRY_CUDA(dq.alloc(128 * 4));
    PP_TRY_CUDA(dsk.alloc(128 * 4));
    PP_TRY_CUDA(dpast.alloc(8));
    PP_TRY_CUDA(dout.alloc(128 * 4));
    PP_TRY_CUDA(cudaMemcpy(dq.p, qdata.data(), 128 * 4, cudaMemcpyHostToDevice));
    PP_TRY_CUDA(cudaMemcpy(dsk.p, scratch.data(), 128 * 4, cudaMemcpyHostToDevice));
    PP_TRY_CUDA(cudaMemcpy(dpast.p, past1, 8, cudaMemcpyHostToDevice));
    PpKvArena a1{};
    a1.struct_size = sizeof a1;
    a1.rows = 2;
    a1.heads = 1;
    a1.head_dim = 64;
    a1.capacity = 3;
    a1.k = a1.v = (uint8_t*)dk.p;
    a1.k_scale = a1.v_scale = (float*)ds.p;
    PP_TRY(run_attention(a1, 32, (const float*)dq.p, (const float*)dsk.p, (const float*)dsk.p,
                         (const uint32_t*)dpast.p, (float*)dout.p));
    std::vector<float> actual(128), rounded(384);
    PP_TRY_CUDA(cudaMemcpy(actual.data(), dout.p, 128 * 4, cudaMemcpyDeviceToHost));
    PP_TRY(pp_b200_dequantize((const uint8_t*)dk.p, (const float*)ds.p, 6, 64, 1, PP_DTYPE_F32, drest.p, nullptr));
    PP_TRY_CUDA(cudaMemcpy(rounded.data(), drest.p, 384 * 4, cudaMemcpyDeviceToHost));
    for (int row = 0; row < 2; ++row) {
        float expect[64];
        expected_row(&qdata[row * 64], &rounded[row * 3 * 64], &rounded[row * 3 * 64], &scratch[row * 64],
                     &scratch[row * 64], past1[row], expect);
        for (int d = 0; d < 64; ++d)
            if (!std::isfinite(actual[row * 64 + d]) || std::fabs(actual[row * 64 + d] - expect[d]) >= 2e-5f)
                return pp::fail_msg(PP_STATUS_PRECONDITION, "KV INT8 attention self-check failed");
    }

    // ---- fixture 2: view offsets, two heads per sequence, empty history,
    // unequal lengths, fixed splits {32, 128} and the automatic stream-K plan.
    const uint32_t rows = 4, cap = 67, heads = 2;
    const size_t n_all = (size_t)(rows + 1) * cap * 64;
    std::vector<float> hist(n_all), vals(n_all);
    for (size_t i = 0; i < n_all; ++i) {
        hist[i] = std::sin((float)i * 0.013f) * 1.7f;
        vals[i] = std::cos((float)i * 0.019f) * 0.8f;
    }
    const size_t row_elems = (size_t)cap * 64;
    DevBuf dh, dv, dkc, dvc, dks, dvs;
    PP_TRY_CUDA(dh.alloc(n_all * 4));
    PP_TRY_CUDA(dv.alloc(n_all * 4));
    PP_TRY_CUDA(dkc.alloc(n_all));
    PP_TRY_CUDA(dvc.alloc(n_all));
    PP_TRY_CUDA(dks.alloc((rows + 1) * cap * 4));
    PP_TRY_CUDA(dvs.alloc((rows + 1) * cap * 4));
    PP_TRY_CUDA(cudaMemcpy(dh.p, hist.data(), n_all * 4, cudaMemcpyHostToDevice));
    PP_TRY_CUDA(cudaMemcpy(dv.p, vals.data(), n_all * 4, cudaMemcpyHostToDevice));
    // Quantize the narrowed views (rows 1..4) straight into rows 1..4 of the
    // (rows+1)-row arenas; row 0 receives a copy of the first quantized row.
    uint8_t* kc1 = (uint8_t*)dkc.p + row_elems;
    uint8_t* vc1 = (uint8_t*)dvc.p + row_elems;
    float* ks1 = (float*)dks.p + cap;
    float* vs1 = (float*)dvs.p + cap;
    PP_TRY(pp_b200_quantize((const float*)dh.p + row_elems, PP_DTYPE_F32, (uint64_t)rows * cap, 64, kc1, ks1, nullptr, nullptr));
    PP_TRY(pp_b200_quantize((const float*)dv.p + row_elems, PP_DTYPE_F32, (uint64_t)rows * cap, 64, vc1, vs1, nullptr, nullptr));
    PP_TRY_CUDA(cudaMemcpy(dkc.p, kc1, row_elems, cudaMemcpyDeviceToDevice));
    PP_TRY_CUDA(cudaMemcpy(dvc.p, vc1, row_elems, cudaMemcpyDeviceToDevice));
    PP_TRY_CUDA(cudaMemcpy(dks.p, ks1, cap * 4, cudaMemcpyDeviceToDevice));
    PP_TRY_CUDA(cudaMemcpy(dvs.p, vs1, cap * 4, cudaMemcpyDeviceToDevice));
    auto vec = [&](float factor, float phase) {
        std::vector<float> v((rows + 1) * 64);
        for (size_t i = 0; i < v.size(); ++i) v[i] = std::sin((float)i * factor + phase);
        return v;
    };
    const std::vector<float> q2 = vec(0.027f, 0.4f), sk2 = vec(0.031f, 1.1f), sv2 = vec(0.047f, -0.8f);
    const uint32_t past_all[3] = {999u, 0u, 66u};
    DevBuf dq2, dsk2, dsv2, dpast2, dout2;
    PP_TRY_CUDA(dq2.alloc(q2.size() * 4));
    PP_TRY_CUDA(dsk2.alloc(sk2.size() * 4));
    PP_TRY_CUDA(dsv2.alloc(sv2.size() * 4));
    PP_TRY_CUDA(dpast2.alloc(12));
    PP_TRY_CUDA(dout2.alloc(rows * 64 * 4));
    PP_TRY_CUDA(cudaMemcpy(dq2.p, q2.data(), q2.size() * 4, cudaMemcpyHostToDevice));
    PP_TRY_CUDA(cudaMemcpy(dsk2.p, sk2.data(), sk2.size() * 4, cudaMemcpyHostToDevice));
    PP_TRY_CUDA(cudaMemcpy(dsv2.p, sv2.data(), sv2.size() * 4, cudaMemcpyHostToDevice));
    PP_TRY_CUDA(cudaMemcpy(dpast2.p, past_all, 12, cudaMemcpyHostToDevice));
    PpKvArena a2{};
    a2.struct_size = sizeof a2;
    a2.rows = rows;
    a2.heads = heads;
    a2.head_dim = 64;
    a2.capacity = cap;
    a2.k = kc1;
    a2.v = vc1;
    a2.k_scale = ks1;
    a2.v_scale = vs1;
    std::vector<float> kcr(rows * row_elems), vcr(rows * row_elems);
    DevBuf dtmp;
    PP_TRY_CUDA(dtmp.alloc(rows * row_elems * 4));
    PP_TRY(pp_b200_dequantize(kc1, ks1, (uint64_t)rows * cap, 64, 1, PP_DTYPE_F32, dtmp.p, nullptr));
    PP_TRY_CUDA(cudaMemcpy(kcr.data(), dtmp.p, rows * row_elems * 4, cudaMemcpyDeviceToHost));
    PP_TRY(pp_b200_dequantize(vc1, vs1, (uint64_t)rows * cap, 64, 1, PP_DTYPE_F32, dtmp.p, nullptr));
    PP_TRY_CUDA(cudaMemcpy(vcr.data(), dtmp.p, rows * row_elems * 4, cudaMemcpyDeviceToHost));
    std::vector<float> reference(rows * 64);
    for (uint32_t row = 0; row < rows; ++row) {
        const uint32_t len = row / heads == 0 ? 0u : 66u;
        expected_row(&q2[(row + 1) * 64], &kcr[row * row_elems], &vcr[row * row_elems], &sk2[(row + 1) * 64],
                     &sv2[(row + 1) * 64], len, &reference[row * 64]);
    }
    const uint32_t splits[3] = {32u, 128u, 0u};
    for (uint32_t split : splits) {
        PP_TRY(run_attention(a2, split, (const float*)dq2.p + 64, (const float*)dsk2.p + 64, (const float*)dsv2.p + 64,
                             (const uint32_t*)dpast2.p + 1, (float*)dout2.p));
        std::vector<float> got(rows * 64);
        PP_TRY_CUDA(cudaMemcpy(got.data(), dout2.p, rows * 64 * 4, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < got.size(); ++i)
            if (!std::isfinite(got[i]) || std::fabs(got[i] - reference[i]) >= 2e-5f)
                return pp::fail_msg(PP_STATUS_PRECONDITION, "KV INT8 offset/split attention self-check failed");
    }
    return PP_STATUS_OK;
}

// prepare_optional_kernels (app/src/model/mod.rs:440-460): zero inputs through
// the fused float attention (and SwiGLU), every output finite and within 1e-6.
int32_t optional_selfcheck(uint32_t fusion, uint32_t split_k, int32_t dtype, uint32_t width, uint32_t ffn_hidden) {
    const size_t elem = dtype == PP_DTYPE_F32 ? 4 : 2;
    DevBuf dq, dk, dv, dout, dws;
    PP_TRY_CUDA(dq.alloc(width * 4));
    PP_TRY_CUDA(dk.alloc(257 * width * elem));
    PP_TRY_CUDA(dv.alloc(257 * width * elem));
    PP_TRY_CUDA(dout.alloc(width * 4));
    PP_TRY_CUDA(cudaMemset(dq.p, 0, width * 4));
    PP_TRY_CUDA(cudaMemset(dk.p, 0, 257 * width * elem));
    PP_TRY_CUDA(cudaMemset(dv.p, 0, 257 * width * elem));
    PpFloatKv kv{};
    kv.struct_size = sizeof kv;
    kv.rows = 1;
    kv.heads = 1;
    kv.head_dim = width;
    kv.tokens = 257;
    kv.dtype = dtype;
    kv.k_row_stride = kv.v_row_stride = 257ull * width;
    kv.k = dk.p;
    kv.v = dv.p;
    PpAttnParams p{};
    p.struct_size = sizeof p;
    p.split_tokens = split_k ? 128u : 0u;
    p.q_dtype = PP_DTYPE_F32;
    p.out_dtype = PP_DTYPE_F32;
    const size_t ws_bytes = pp_b200_float_attention_workspace_size(&kv, &p);
    PP_TRY_CUDA(dws.alloc(ws_bytes));
    PP_TRY(pp_b200_decode_attention_float(&kv, &p, dq.p, width, nullptr, dout.p, dws.p, ws_bytes, nullptr, nullptr));
    PP_TRY_CUDA(cudaDeviceSynchronize());
    std::vector<float> got(width);
    PP_TRY_CUDA(cudaMemcpy(got.data(), dout.p, width * 4, cudaMemcpyDeviceToHost));
    for (float x : got)
        if (!std::isfinite(x) || std::fabs(x) > 1e-6f)
            return pp::fail_msg(PP_STATUS_PRECONDITION, "融合注意力准备验证失败");
    if (fusion) {
        const uint64_t n = 2ull * ffn_hidden;
        DevBuf dg, dh;
        PP_TRY_CUDA(dg.alloc(n * elem));
        PP_TRY_CUDA(dh.alloc(ffn_hidden * elem));
        PP_TRY_CUDA(cudaMemset(dg.p, 0, n * elem));
        PP_TRY(pp_b200_swiglu(dg.p, dh.p, 1, ffn_hidden, dtype, nullptr));
        PP_TRY_CUDA(cudaDeviceSynchronize());
        std::vector<float> h(ffn_hidden);
        if (dtype == PP_DTYPE_F32) {
            PP_TRY_CUDA(cudaMemcpy(h.data(), dh.p, ffn_hidden * 4, cudaMemcpyDeviceToHost));
        } else {
            std::vector<uint16_t> b(ffn_hidden);
            PP_TRY_CUDA(cudaMemcpy(b.data(), dh.p, ffn_hidden * 2, cudaMemcpyDeviceToHost));
            for (uint32_t i = 0; i < ffn_hidden; ++i) {
                const uint32_t u = (uint32_t)b[i] << 16;
                std::memcpy(&h[i], &u, 4);
            }
        }
        for (float x : h)
            if (!std::isfinite(x) || std::fabs(x) > 1e-6f) return pp::fail_msg(PP_STATUS_PRECONDITION, "融合FFN准备验证失败");
    }
    return PP_STATUS_OK;
}

}  // namespace

extern "C" int32_t pp_b200_prepare_optional(int32_t device, uint32_t fusion, uint32_t split_k, int32_t model_dtype,
                                            uint32_t head_width, uint32_t ffn_hidden) {
    if (!fusion && !split_k) return PP_STATUS_OK;
    if ((head_width != 64 && head_width != 128) || (model_dtype != PP_DTYPE_F32 && model_dtype != PP_DTYPE_BF16) ||
        (fusion && ffn_hidden == 0))
        return pp::fail_msg(PP_STATUS_PRECONDITION, "当前模型后端不支持此融合解码路径");
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return pp::fail_msg(PP_STATUS_PRECONDITION, "当前模型后端不支持此融合解码路径");
    if ((e = cudaSetDevice(device)) != cudaSuccess)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "当前模型后端不支持此融合解码路径");
    const int32_t s = optional_selfcheck(fusion, split_k, model_dtype, head_width, ffn_hidden);
    cudaSetDevice(prev);
    return s;
}

extern "C" int32_t pp_b200_prepare(int32_t device) {
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return pp::fail_msg(PP_STATUS_PRECONDITION, "KV INT8 needs CUDA in the native provider");
    if ((e = cudaSetDevice(device)) != cudaSuccess)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "KV INT8 needs CUDA in the native provider: invalid device");
    const int32_t s = selfcheck();
    cudaSetDevice(prev);
    return s;
}
