// SPDX-License-Identifier: MIT
//
// _C_cuda: CUDA implementations of the seven torch.ops.beamgrad operators
// (schemas of beamgrad 2.3.0, python/csrc/cpu_ops.cpp:582-608), on this
// engine's C ABI (include/dbs_cuda.h). A drop-in for beamgrad's own _C_cuda
// (python/csrc/cuda_ops.cpp): same operator names, argument meaning, output
// shapes and dtypes, ValueError for bad arguments, RuntimeError for engine
// failures, and the module functions device_available() / max_beam_size().
//
// Work is enqueued on PyTorch's current stream; outputs and scratch come from
// PyTorch's caching allocator. Host read-backs (hence synchronizations) happen
// only where the operator semantics need them: validating per-example steps,
// and validate=true (the NaN/+inf flags, plus the equal-length check of
// decode_step).
#include <Python.h>

#include <torch/all.h>
#include <torch/library.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <cmath>
#include <limits>
#include <tuple>
#include <vector>

#include "dbs_cuda.h"
#include "dbs_cuda_b200.h"

namespace {

using at::Tensor;
using OptTensor = c10::optional<Tensor>;
constexpr int64_t kInt32Max = std::numeric_limits<int32_t>::max();

cudaStream_t current_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Engine status -> Python exception (ValueError for arguments, RuntimeError otherwise).
void raise_on(int status, const char* op) {
    TORCH_CHECK_VALUE(status != DBS_CUDA_STATUS_INVALID_ARGUMENT, "beamgrad CUDA ", op, ": invalid argument");
    TORCH_CHECK(status == DBS_CUDA_STATUS_OK, "beamgrad CUDA ", op, " failed: ", dbs_cuda_status_string(status));
}

void need_extent(int64_t n, const char* what) {
    TORCH_CHECK_VALUE(n >= 1 && n <= kInt32Max, what, " must be in [1, INT_MAX], got ", n);
}

void need_penalties(double alpha, double repetition) {
    TORCH_CHECK_VALUE(std::isfinite(alpha) && alpha >= 0.0, "length_penalty_alpha must be finite and non-negative");
    TORCH_CHECK_VALUE(std::isfinite(repetition) && repetition > 0.0, "repetition_penalty must be finite and positive");
}

int engine_dtype(const Tensor& t, const char* what) {
    if (t.scalar_type() == torch::kFloat32) return DBS_CUDA_DTYPE_F32;
    if (t.scalar_type() == torch::kFloat16) return DBS_CUDA_DTYPE_F16;
    if (t.scalar_type() == torch::kBFloat16) return DBS_CUDA_DTYPE_BF16;
    TORCH_CHECK_VALUE(false, what, " must be float32, float16 or bfloat16, got ", t.scalar_type());
    return DBS_CUDA_DTYPE_F32;
}

// Per-example step counts: integer [B], each in [1, T]; returned as contiguous int32 on
// `device`. The range is checked on 64-bit values (one flag read back) before narrowing.
OptTensor steps_on_device(const OptTensor& steps, const c10::Device& device, int64_t B, int64_t T) {
    if (!steps.has_value()) return c10::nullopt;
    const Tensor& s = *steps;
    TORCH_CHECK_VALUE(s.dim() == 1 && s.size(0) == B, "steps must have shape [B] = [", B, "]");
    TORCH_CHECK_VALUE(c10::isIntegralType(s.scalar_type(), /*includeBool=*/false),
                      "steps must be an integer tensor, got ", s.scalar_type());
    const Tensor wide = s.to(device, torch::kInt64);
    const bool in_range = wide.ge(1).logical_and(wide.le(T)).all().item<bool>();
    if (!in_range) {
        const Tensor host = wide.cpu();
        const auto* v = host.data_ptr<int64_t>();
        for (int64_t b = 0; b < B; ++b)
            TORCH_CHECK_VALUE(v[b] >= 1 && v[b] <= T, "steps[", b, "] = ", v[b], " must be in [1, ", T, "]");
    }
    return wide.to(torch::kInt32).contiguous();
}

// The engine's problem description; steps (if any) already validated on the device.
DBSCudaDecodeArgs problem(int64_t B, int64_t T, int64_t K, int64_t V, int64_t eos, int64_t min_length, double alpha,
                          const OptTensor& steps_i32) {
    need_extent(B, "B");
    need_extent(T, "T");
    need_extent(K, "K");
    need_extent(V, "V");
    TORCH_CHECK_VALUE(K <= DBS_CUDA_MAX_BEAM, "beam_size ", K, " exceeds the CUDA backend maximum of ", DBS_CUDA_MAX_BEAM);
    TORCH_CHECK_VALUE(eos >= -1 && eos < V, "eos_token must be -1 or a token id < ", V);
    TORCH_CHECK_VALUE(min_length >= 0 && min_length <= kInt32Max, "min_length must be non-negative");
    DBSCudaDecodeArgs a{};
    a.batch_size = static_cast<int>(B);
    a.steps = static_cast<int>(T);
    a.beam_size = static_cast<int>(K);
    a.vocab_size = static_cast<int>(V);
    a.eos_token = static_cast<int>(eos);
    a.min_length = static_cast<int>(min_length);
    a.length_penalty_alpha = static_cast<float>(alpha);
    a.repetition_penalty = 1.0f;
    if (steps_i32.has_value()) a.steps_per_example = steps_i32->data_ptr<int32_t>();
    return a;
}

// Constraint arguments shared by the decode operators. `keep` owns the banned mask.
void constraints(DBSCudaDecodeArgs& a, const OptTensor& banned_tokens, int64_t ngram, double repetition,
                 const c10::Device& device, Tensor& keep) {
    a.no_repeat_ngram_size = static_cast<int>(std::clamp<int64_t>(ngram, 0, kInt32Max));
    a.repetition_penalty = static_cast<float>(repetition);
    if (!banned_tokens.has_value()) return;
    keep = banned_tokens->to(device, torch::kUInt8).contiguous();
    TORCH_CHECK_VALUE(keep.dim() == 1 && keep.size(0) == a.vocab_size, "banned_tokens must be a [V] mask");
    a.banned_tokens = keep.data_ptr<uint8_t>();
}

DBSCudaSearchOptions extra_eos_options(c10::IntArrayRef extra_eos, int64_t eos, int64_t V) {
    TORCH_CHECK_VALUE(static_cast<int64_t>(extra_eos.size()) <= DBS_CUDA_MAX_EXTRA_EOS, "at most ",
                      DBS_CUDA_MAX_EXTRA_EOS, " extra EOS tokens are supported on CUDA, got ", extra_eos.size());
    TORCH_CHECK_VALUE(extra_eos.empty() || eos >= 0, "extra EOS tokens need eos_token >= 0");
    DBSCudaSearchOptions o{};
    for (int64_t tok : extra_eos) {
        TORCH_CHECK_VALUE(tok >= 0 && tok < V, "extra EOS token ", tok, " is outside the vocabulary (size ", V, ")");
        o.extra_eos_tokens[o.extra_eos_count++] = static_cast<int32_t>(tok);
    }
    return o;
}

Tensor scratch(int64_t bytes, const Tensor& like) {
    TORCH_CHECK_VALUE(bytes >= 0, "beamgrad CUDA: unsupported problem size (see DBS_CUDA_MAX_BEAM and the limits in dbs_cuda.h)");
    return torch::empty({std::max<int64_t>(bytes, 1)}, like.options().dtype(torch::kUInt8));
}

// The trace tensors [B, T, K] of a decode, and the engine's view of them.
struct Trace {
    Tensor final_scores, final_raw, final_lengths, tokens, parents, lengths, scores, raw_scores, from_logprob, row_lse,
        invalid;
    DBSCudaDecodeOutputs view{};

    Trace(const Tensor& like, int64_t B, int64_t T, int64_t K, bool validate) {
        const auto f32 = like.options().dtype(torch::kFloat32);
        const auto i32 = like.options().dtype(torch::kInt32);
        const auto u8 = like.options().dtype(torch::kUInt8);
        final_scores = torch::empty({B, K}, f32);
        final_raw = torch::empty({B, K}, f32);
        final_lengths = torch::empty({B, K}, i32);
        tokens = torch::empty({B, T, K}, i32);
        parents = torch::empty({B, T, K}, i32);
        lengths = torch::empty({B, T, K}, i32);
        scores = torch::empty({B, T, K}, f32);
        raw_scores = torch::empty({B, T, K}, f32);
        from_logprob = torch::empty({B, T, K}, u8);
        row_lse = torch::empty({B, T, K}, f32);
        if (validate) invalid = torch::empty({B}, u8);
        view.final_scores = final_scores.data_ptr<float>();
        view.final_raw_scores = final_raw.data_ptr<float>();
        view.final_lengths = final_lengths.data_ptr<int32_t>();
        view.tokens = tokens.data_ptr<int32_t>();
        view.parents = parents.data_ptr<int32_t>();
        view.lengths = lengths.data_ptr<int32_t>();
        view.scores = scores.data_ptr<float>();
        view.raw_scores = raw_scores.data_ptr<float>();
        view.from_logprob = from_logprob.data_ptr<uint8_t>();
        view.invalid_input = validate ? invalid.data_ptr<uint8_t>() : nullptr;
    }
};

// validate=true: one byte per example read back (synchronizes the stream).
void reject_flagged(const Tensor& invalid, const char* what) {
    const Tensor host = invalid.cpu();
    const auto* f = host.data_ptr<uint8_t>();
    for (int64_t b = 0; b < host.numel(); ++b)
        TORCH_CHECK_VALUE(f[b] == 0, "example ", b, ": ", what, " NaN or +inf in a row the search reads");
}

using DecodeExResult = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;
using DecodeResult = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;
using StepResult = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;

DecodeExResult op_decode_ex(const Tensor& inputs, bool from_logits, const OptTensor& steps, int64_t eos_token,
                            int64_t min_length, double length_penalty_alpha, const OptTensor& banned_tokens,
                            int64_t no_repeat_ngram_size, double repetition_penalty, bool validate,
                            c10::IntArrayRef extra_eos) {
    TORCH_CHECK(inputs.is_cuda(), "beamgrad::decode (CUDA) expects a CUDA tensor");
    const int dtype = engine_dtype(inputs, from_logits ? "logits" : "log_probs");
    TORCH_CHECK_VALUE(inputs.dim() == 4, "inputs must have shape [B, T, K, V]");
    need_penalties(length_penalty_alpha, repetition_penalty);
    const c10::cuda::CUDAGuard guard(inputs.device());
    const Tensor x = inputs.contiguous();
    const int64_t B = x.size(0), T = x.size(1), K = x.size(2), V = x.size(3);
    const OptTensor steps_i32 = steps_on_device(steps, x.device(), B, T);
    DBSCudaDecodeArgs args = problem(B, T, K, V, eos_token, min_length, length_penalty_alpha, steps_i32);
    Tensor banned;
    constraints(args, banned_tokens, no_repeat_ngram_size, repetition_penalty, x.device(), banned);
    const DBSCudaSearchOptions opts = extra_eos_options(extra_eos, eos_token, V);
    Trace tr(x, B, T, K, validate);
    const int64_t ws_bytes = dbs_cuda_decode_workspace_size(&args);
    Tensor ws = scratch(ws_bytes, x);
    raise_on(dbs_cuda_decode_ex2(x.data_ptr(), dtype, from_logits ? 1 : 0, &args, &opts, &tr.view,
                                 tr.row_lse.data_ptr<float>(), ws.data_ptr(), ws_bytes, current_stream()),
             "decode");
    if (validate) reject_flagged(tr.invalid, from_logits ? "logits contain" : "log_probs contains");
    return {tr.final_scores, tr.final_raw, tr.final_lengths, tr.tokens, tr.parents,
            tr.lengths,      tr.scores,    tr.raw_scores,    tr.from_logprob, tr.row_lse};
}

DecodeResult op_decode(const Tensor& log_probs, const OptTensor& steps, int64_t eos_token, int64_t min_length,
                       double length_penalty_alpha, const OptTensor& banned_tokens, int64_t no_repeat_ngram_size,
                       double repetition_penalty, bool validate) {
    TORCH_CHECK_VALUE(log_probs.scalar_type() == torch::kFloat32, "log_probs must be float32");
    auto r = op_decode_ex(log_probs, false, steps, eos_token, min_length, length_penalty_alpha, banned_tokens,
                          no_repeat_ngram_size, repetition_penalty, validate, {});
    return {std::get<0>(r), std::get<1>(r), std::get<2>(r), std::get<3>(r), std::get<4>(r),
            std::get<5>(r), std::get<6>(r), std::get<7>(r), std::get<8>(r)};
}

StepResult op_decode_step(const Tensor& log_probs, const Tensor& raw_scores, const Tensor& lengths,
                          const Tensor& finished, const Tensor& prefixes, int64_t eos_token, int64_t min_length,
                          double length_penalty_alpha, const OptTensor& banned_tokens, int64_t no_repeat_ngram_size,
                          double repetition_penalty, bool validate, c10::IntArrayRef extra_eos) {
    TORCH_CHECK(log_probs.is_cuda(), "beamgrad::decode_step (CUDA) expects CUDA tensors");
    TORCH_CHECK_VALUE(log_probs.scalar_type() == torch::kFloat32 && log_probs.dim() == 3,
                      "log_probs must be a float32 [B, K, V] tensor");
    const c10::cuda::CUDAGuard guard(log_probs.device());
    const Tensor x = log_probs.contiguous();
    const int64_t B = x.size(0), K = x.size(1), V = x.size(2);
    for (const Tensor* t : {&raw_scores, &lengths, &finished, &prefixes})
        TORCH_CHECK_VALUE(t->device() == x.device(), "the beam state must be on the device of log_probs");
    const std::vector<int64_t> bk{B, K};
    TORCH_CHECK_VALUE(raw_scores.scalar_type() == torch::kFloat32 && raw_scores.sizes() == c10::IntArrayRef(bk),
                      "raw_scores must be a float32 [B, K] tensor");
    TORCH_CHECK_VALUE(lengths.scalar_type() == torch::kInt32 && lengths.sizes() == c10::IntArrayRef(bk),
                      "lengths must be an int32 [B, K] tensor");
    TORCH_CHECK_VALUE(finished.scalar_type() == torch::kUInt8 && finished.sizes() == c10::IntArrayRef(bk),
                      "finished must be a uint8 [B, K] tensor");
    TORCH_CHECK_VALUE(prefixes.scalar_type() == torch::kInt32 && prefixes.dim() == 3 && prefixes.size(0) == B &&
                          prefixes.size(1) == K && prefixes.size(2) <= kInt32Max,
                      "prefixes must be an int32 [B, K, L] tensor");
    need_penalties(length_penalty_alpha, repetition_penalty);
    DBSCudaDecodeArgs args = problem(B, 1, K, V, eos_token, min_length, length_penalty_alpha, c10::nullopt);
    Tensor banned;
    constraints(args, banned_tokens, no_repeat_ngram_size, repetition_penalty, x.device(), banned);
    const DBSCudaSearchOptions opts = extra_eos_options(extra_eos, eos_token, V);

    // The engine advances the state in place: work on copies, leave the inputs as they are.
    Tensor raw = raw_scores.contiguous().clone();
    Tensor len = lengths.contiguous().clone();
    Tensor fin = finished.contiguous().clone();
    const Tensor pre = prefixes.contiguous();
    const auto i32 = x.options().dtype(torch::kInt32);
    Tensor tokens = torch::empty({B, K}, i32);
    Tensor parents = torch::empty({B, K}, i32);
    Tensor scores = torch::empty({B, K}, x.options());
    Tensor final_scores = torch::empty({B, K}, x.options());
    Tensor from_logprob = torch::empty({B, K}, x.options().dtype(torch::kUInt8));
    Tensor invalid = validate ? torch::empty({B}, x.options().dtype(torch::kUInt8)) : Tensor();

    // Candidates are ranked by raw score, which matches the CPU decoder's ranking by
    // penalised score when the live, unfinished beams of an example share one length
    // (always true of states the search produces). With validation that precondition is
    // checked on the device and read back together with the NaN flags.
    Tensor span;
    if (validate && length_penalty_alpha != 0.0) {
        Tensor extended = torch::isfinite(raw_scores);
        if (eos_token >= 0) extended = extended.logical_and(finished.eq(0));
        const Tensor lo = torch::where(extended, lengths, torch::full_like(lengths, kInt32Max)).amin(1);
        const Tensor hi = torch::where(extended, lengths, torch::full_like(lengths, -1)).amax(1);
        span = torch::stack({lo, hi});
    }

    DBSCudaDecodeOutputs out{};
    out.tokens = tokens.data_ptr<int32_t>();
    out.parents = parents.data_ptr<int32_t>();
    out.scores = scores.data_ptr<float>();
    out.from_logprob = from_logprob.data_ptr<uint8_t>();
    out.final_scores = final_scores.data_ptr<float>();
    out.invalid_input = validate ? invalid.data_ptr<uint8_t>() : nullptr;
    DBSCudaBeamState state{};
    state.raw_scores = raw.data_ptr<float>();
    state.lengths = len.data_ptr<int32_t>();
    state.finished = fin.data_ptr<uint8_t>();
    state.prefixes = pre.numel() > 0 ? pre.data_ptr<int32_t>() : nullptr;
    state.prefix_stride = static_cast<int>(pre.size(2));
    const int64_t ws_bytes = dbs_cuda_decode_step_workspace_size(&args, state.prefix_stride);
    Tensor ws = scratch(ws_bytes, x);
    raise_on(dbs_cuda_decode_step_ex2(x.data_ptr<float>(), DBS_CUDA_DTYPE_F32, 0, &args, &opts, &state, &out, nullptr,
                                      ws.data_ptr(), ws_bytes, current_stream()),
             "decode_step");
    if (validate) {
        Tensor host = invalid.to(torch::kInt32).unsqueeze(0);
        if (span.defined()) host = torch::cat({host, span});
        host = host.cpu();
        const auto* h = host.data_ptr<int32_t>();
        if (span.defined()) {
            for (int64_t b = 0; b < B; ++b)
                TORCH_CHECK_VALUE(h[2 * B + b] <= h[B + b], "example ", b,
                                  ": with length_penalty_alpha != 0, decode_step on CUDA needs every live, unfinished "
                                  "beam to have the same length (as in any state the search produced), got lengths "
                                  "from ", h[B + b], " to ", h[2 * B + b]);
        }
        for (int64_t b = 0; b < B; ++b)
            TORCH_CHECK_VALUE(h[b] == 0, "example ", b, ": log_probs contains NaN or +inf in a row the search reads");
    }
    return {tokens, parents, len, scores, raw, from_logprob, fin, final_scores};
}

// The trace of a decode handed to the backward operators, checked and made contiguous.
struct TraceIn {
    Tensor parents, tokens, lengths, from_logprob;
    int64_t B, T, K;

    TraceIn(const Tensor& par, const Tensor& tok, const Tensor& len, const Tensor& flp, const char* op) {
        TORCH_CHECK(par.is_cuda(), "beamgrad::", op, " (CUDA) expects CUDA tensors");
        TORCH_CHECK_VALUE(par.dim() == 3 && par.scalar_type() == torch::kInt32, "parents must be an int32 [B, T, K] tensor");
        B = par.size(0);
        T = par.size(1);
        K = par.size(2);
        for (const Tensor* t : {&tok, &len})
            TORCH_CHECK_VALUE(t->device() == par.device() && t->sizes() == par.sizes() && t->scalar_type() == torch::kInt32,
                              "tokens and lengths must be int32 [B, T, K] tensors on the same device");
        TORCH_CHECK_VALUE(flp.device() == par.device() && flp.sizes() == par.sizes() && flp.scalar_type() == torch::kUInt8,
                          "from_logprob must be a uint8 [B, T, K] tensor on the same device");
        parents = par.contiguous();
        tokens = tok.contiguous();
        lengths = len.contiguous();
        from_logprob = flp.contiguous();
    }
};

Tensor final_grad_checked(const Tensor& g, const TraceIn& tr) {
    TORCH_CHECK_VALUE(g.device() == tr.parents.device() && g.scalar_type() == torch::kFloat32 && g.dim() == 2 &&
                          g.size(0) == tr.B && g.size(1) == tr.K,
                      "grad_final must be a float32 [B, K] tensor on the same device");
    return g.contiguous();
}

Tensor op_final_scores_backward(const Tensor& grad_final, const Tensor& parents, const Tensor& tokens,
                                const Tensor& lengths, const Tensor& from_logprob, const OptTensor& steps,
                                int64_t vocab_size, double length_penalty_alpha) {
    const TraceIn tr(parents, tokens, lengths, from_logprob, "final_scores_backward");
    const c10::cuda::CUDAGuard guard(tr.parents.device());
    const Tensor g = final_grad_checked(grad_final, tr);
    const OptTensor steps_i32 = steps_on_device(steps, tr.parents.device(), tr.B, tr.T);
    const DBSCudaDecodeArgs args = problem(tr.B, tr.T, tr.K, vocab_size, -1, 0, length_penalty_alpha, steps_i32);
    // One write pass (dbs_cuda_backward_dense) instead of a zero-fill plus the scatter.
    DBSCudaBackwardInputs in{};
    in.parents = tr.parents.data_ptr<int32_t>();
    in.tokens = tr.tokens.data_ptr<int32_t>();
    in.lengths = tr.lengths.data_ptr<int32_t>();
    in.from_logprob = tr.from_logprob.data_ptr<uint8_t>();
    in.grad_final_scores = g.data_ptr<float>();
    Tensor grad = torch::empty({tr.B, tr.T, tr.K, vocab_size}, g.options());
    const int64_t ws_bytes = dbs_cuda_backward_workspace_size(&args);
    const Tensor ws = scratch(ws_bytes, tr.parents);
    raise_on(dbs_cuda_backward_dense(&args, &in, grad.data_ptr(), DBS_CUDA_DTYPE_F32, ws.data_ptr(), ws_bytes,
                                     current_stream()),
             "backward");
    return grad;
}

Tensor op_final_scores_path_gradient(const Tensor& grad_final, const Tensor& parents, const Tensor& tokens,
                                     const Tensor& lengths, const Tensor& from_logprob, const OptTensor& steps,
                                     int64_t vocab_size, double length_penalty_alpha) {
    const TraceIn tr(parents, tokens, lengths, from_logprob, "final_scores_path_gradient");
    const c10::cuda::CUDAGuard guard(tr.parents.device());
    const Tensor g = final_grad_checked(grad_final, tr);
    const OptTensor steps_i32 = steps_on_device(steps, tr.parents.device(), tr.B, tr.T);
    const DBSCudaDecodeArgs args = problem(tr.B, tr.T, tr.K, vocab_size, -1, 0, length_penalty_alpha, steps_i32);
    Tensor draws = torch::empty({tr.B, tr.T, tr.K}, g.options());
    raise_on(dbs_cuda_path_gradient(&args, tr.parents.data_ptr<int32_t>(), tr.tokens.data_ptr<int32_t>(),
                                    tr.lengths.data_ptr<int32_t>(), tr.from_logprob.data_ptr<uint8_t>(),
                                    g.data_ptr<float>(), draws.data_ptr<float>(), current_stream()),
             "path gradient");
    return draws;
}

// An optional score gradient of the given shape (float32, on `device`); null when absent.
const float* score_grad(const OptTensor& g, c10::IntArrayRef shape, const c10::Device& device, const char* name,
                        Tensor& keep) {
    if (!g.has_value()) return nullptr;
    TORCH_CHECK_VALUE(g->device() == device && g->scalar_type() == torch::kFloat32 && g->sizes() == shape, name,
                      " must be a float32 ", shape, " tensor on the device of the trace");
    keep = g->contiguous();
    return keep.data_ptr<float>();
}

// The dense input gradient of a decode in `out_type`, written in one pass by
// dbs_cuda_backward_dense: identical to zero-filling a float32 gradient,
// accumulating the backward into it and casting the result to out_type.
Tensor decode_backward_impl(const OptTensor& grad_final_scores, const OptTensor& grad_final_raw_scores,
                            const OptTensor& grad_scores, const OptTensor& grad_raw_scores, const Tensor& parents,
                            const Tensor& tokens, const Tensor& lengths, const Tensor& from_logprob,
                            const OptTensor& steps, int64_t vocab_size, double length_penalty_alpha,
                            const OptTensor& logits, const OptTensor& row_lse, c10::ScalarType out_type) {
    const TraceIn tr(parents, tokens, lengths, from_logprob, "decode_backward");
    const c10::cuda::CUDAGuard guard(tr.parents.device());
    const c10::Device device = tr.parents.device();
    const std::vector<int64_t> bk{tr.B, tr.K}, btk{tr.B, tr.T, tr.K};
    Tensor k_final, k_final_raw, k_scores, k_raw, x, lse;
    DBSCudaBackwardInputs in{};
    in.grad_final_scores = score_grad(grad_final_scores, bk, device, "grad_final_scores", k_final);
    in.grad_final_raw_scores = score_grad(grad_final_raw_scores, bk, device, "grad_final_raw_scores", k_final_raw);
    in.grad_scores = score_grad(grad_scores, btk, device, "grad_scores", k_scores);
    in.grad_raw_scores = score_grad(grad_raw_scores, btk, device, "grad_raw_scores", k_raw);
    in.parents = tr.parents.data_ptr<int32_t>();
    in.tokens = tr.tokens.data_ptr<int32_t>();
    in.lengths = tr.lengths.data_ptr<int32_t>();
    in.from_logprob = tr.from_logprob.data_ptr<uint8_t>();
    TORCH_CHECK_VALUE(logits.has_value() == row_lse.has_value(), "logits and row_lse must be given together");
    if (logits.has_value()) {
        in.logits_type = engine_dtype(*logits, "logits");
        TORCH_CHECK_VALUE(logits->device() == device && logits->dim() == 4 && logits->size(0) == tr.B &&
                              logits->size(1) == tr.T && logits->size(2) == tr.K && logits->size(3) == vocab_size,
                          "logits must be a [B, T, K, V] = [", tr.B, ", ", tr.T, ", ", tr.K, ", ", vocab_size,
                          "] tensor on the same device");
        TORCH_CHECK_VALUE(row_lse->device() == device && row_lse->scalar_type() == torch::kFloat32 &&
                              row_lse->sizes() == c10::IntArrayRef(btk),
                          "row_lse must be a float32 [B, T, K] tensor on the same device");
        x = logits->contiguous();
        lse = row_lse->contiguous();
        in.logits = x.data_ptr();
        in.row_lse = lse.data_ptr<float>();
    }
    const OptTensor steps_i32 = steps_on_device(steps, device, tr.B, tr.T);
    const DBSCudaDecodeArgs args = problem(tr.B, tr.T, tr.K, vocab_size, -1, 0, length_penalty_alpha, steps_i32);
    int grad_type = DBS_CUDA_DTYPE_F32;
    if (out_type == torch::kFloat16) grad_type = DBS_CUDA_DTYPE_F16;
    else if (out_type == torch::kBFloat16) grad_type = DBS_CUDA_DTYPE_BF16;
    else TORCH_CHECK_VALUE(out_type == torch::kFloat32, "the gradient dtype must be float32, float16 or bfloat16");
    Tensor grad = torch::empty({tr.B, tr.T, tr.K, vocab_size}, tr.parents.options().dtype(out_type));
    const int64_t ws_bytes = dbs_cuda_backward_workspace_size(&args);
    const Tensor ws = scratch(ws_bytes, tr.parents);
    raise_on(dbs_cuda_backward_dense(&args, &in, grad.data_ptr(), grad_type, ws.data_ptr(), ws_bytes, current_stream()),
             "backward");
    return grad;
}

Tensor op_decode_backward(const OptTensor& grad_final_scores, const OptTensor& grad_final_raw_scores,
                          const OptTensor& grad_scores, const OptTensor& grad_raw_scores, const Tensor& parents,
                          const Tensor& tokens, const Tensor& lengths, const Tensor& from_logprob,
                          const OptTensor& steps, int64_t vocab_size, double length_penalty_alpha,
                          const OptTensor& logits, const OptTensor& row_lse) {
    return decode_backward_impl(grad_final_scores, grad_final_raw_scores, grad_scores, grad_raw_scores, parents, tokens,
                                lengths, from_logprob, steps, vocab_size, length_penalty_alpha, logits, row_lse,
                                torch::kFloat32);
}

// beamgrad_b200::decode_backward_as: decode_backward with the gradient written
// directly in `dtype` (the input's dtype in autograd), replacing
// decode_backward(...).to(dtype) (python/beamgrad/_torch.py:289 of beamgrad 2.3.0).
Tensor op_decode_backward_as(const OptTensor& grad_final_scores, const OptTensor& grad_final_raw_scores,
                             const OptTensor& grad_scores, const OptTensor& grad_raw_scores, const Tensor& parents,
                             const Tensor& tokens, const Tensor& lengths, const Tensor& from_logprob,
                             const OptTensor& steps, int64_t vocab_size, double length_penalty_alpha,
                             const OptTensor& logits, const OptTensor& row_lse, c10::ScalarType dtype) {
    return decode_backward_impl(grad_final_scores, grad_final_raw_scores, grad_scores, grad_raw_scores, parents, tokens,
                                lengths, from_logprob, steps, vocab_size, length_penalty_alpha, logits, row_lse, dtype);
}

Tensor op_length_penalty(const Tensor& lengths, double alpha) {
    TORCH_CHECK(lengths.is_cuda(), "beamgrad::length_penalty (CUDA) expects a CUDA tensor");
    TORCH_CHECK_VALUE(c10::isIntegralType(lengths.scalar_type(), /*includeBool=*/false), "lengths must be an integer tensor");
    TORCH_CHECK_VALUE(std::isfinite(alpha) && alpha >= 0.0, "length_penalty_alpha must be finite and non-negative");
    const c10::cuda::CUDAGuard guard(lengths.device());
    const Tensor len = lengths.clamp(0, kInt32Max).to(torch::kInt32).contiguous();
    Tensor out = torch::empty(len.sizes(), len.options().dtype(torch::kFloat32));
    raise_on(dbs_cuda_length_penalty(len.data_ptr<int32_t>(), len.numel(), static_cast<float>(alpha),
                                     out.data_ptr<float>(), current_stream()),
             "length penalty");
    return out;
}

}  // namespace

TORCH_LIBRARY_IMPL(beamgrad, CUDA, m) {
    m.impl("decode", &op_decode);
    m.impl("decode_ex", &op_decode_ex);
    m.impl("decode_step", &op_decode_step);
    m.impl("final_scores_backward", &op_final_scores_backward);
    m.impl("final_scores_path_gradient", &op_final_scores_path_gradient);
    m.impl("decode_backward", &op_decode_backward);
    m.impl("length_penalty", &op_length_penalty);
}

// Operators this engine adds (no counterpart in beamgrad).
TORCH_LIBRARY(beamgrad_b200, m) {
    m.def("decode_backward_as(Tensor? grad_final_scores, Tensor? grad_final_raw_scores, Tensor? grad_scores, "
          "Tensor? grad_raw_scores, Tensor parents, Tensor tokens, Tensor lengths, Tensor from_logprob, Tensor? steps, "
          "int vocab_size, float length_penalty_alpha, Tensor? logits, Tensor? row_lse, ScalarType dtype) -> Tensor");
}

TORCH_LIBRARY_IMPL(beamgrad_b200, CUDA, m) { m.impl("decode_backward_as", &op_decode_backward_as); }

namespace {

PyObject* py_device_available(PyObject*, PyObject*) { return PyBool_FromLong(dbs_cuda_available() != 0); }
PyObject* py_max_beam_size(PyObject*, PyObject*) { return PyLong_FromLong(DBS_CUDA_MAX_BEAM); }

PyMethodDef kMethods[] = {
    {"device_available", py_device_available, METH_NOARGS, "Whether the CUDA runtime reports a usable device"},
    {"max_beam_size", py_max_beam_size, METH_NOARGS, "Largest beam size the CUDA engine supports"},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_C_cuda",
                       "CUDA kernels of the beamgrad operators (torch.ops.beamgrad.*) on the B200 engine", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__C_cuda(void) { return PyModule_Create(&kModule); }
