// SPDX-License-Identifier: MIT
//
// _C_cuda: the seven torch.ops.beamgrad operators on CUDA tensors, running this engine
// through its C ABI (include/dbs_cuda.h), plus beamgrad_b200::decode_backward_as.
//
// The operator contract is beamgrad 2.3.0's: schemas from python/csrc/cpu_ops.cpp:582-608,
// output shapes and dtypes (int32 trace, uint8 flags, float32 scores), ValueError for bad
// arguments, RuntimeError for engine failures, and the module functions
// device_available() / max_beam_size() (python/csrc/cuda_ops.cpp:494-513).
//
// Organisation:
//   * every operator states its argument requirements as a table of rules, checked by one
//     routine (enforce);
//   * every trace tensor an operator returns comes from one output table (TraceOut), which
//     also fills the engine's output struct;
//   * every host read-back an operator needs (the range of per-example steps, NaN/+inf
//     flags, the equal-length precondition of decode_step) is queued in a HostCheck and
//     read in one device-to-host copy.
// Work runs on PyTorch's current stream; outputs and scratch come from PyTorch's allocator.
#include <Python.h>

#include <torch/all.h>
#include <torch/library.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
#include <functional>
#include <initializer_list>
#include <limits>
#include <string>
#include <tuple>
#include <vector>

#include "dbs_cuda.h"
#include "dbs_cuda_b200.h"

namespace {

using at::Tensor;
using OptTensor = c10::optional<Tensor>;
constexpr int64_t kIntMax = std::numeric_limits<int32_t>::max();

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// ---------------------------------------------------------------------------
// Argument rules
// ---------------------------------------------------------------------------

// Element types a tensor argument may have.
enum class Elems { F32, I32, U8, AnyInt, AnyFloat };

bool elems_ok(const Tensor& t, Elems e) {
    const auto s = t.scalar_type();
    switch (e) {
        case Elems::F32: return s == torch::kFloat32;
        case Elems::I32: return s == torch::kInt32;
        case Elems::U8: return s == torch::kUInt8;
        case Elems::AnyInt: return c10::isIntegralType(s, /*includeBool=*/false);
        case Elems::AnyFloat: return s == torch::kFloat32 || s == torch::kFloat16 || s == torch::kBFloat16;
    }
    return false;
}

// One requirement of an operator. A tensor rule checks element type, shape (-1: any extent)
// and, when `device` is set, the device; a plain rule is a precomputed condition. A failed
// rule raises ValueError with `says`.
struct Rule {
    const Tensor* t = nullptr;
    Elems elems = Elems::F32;
    std::vector<int64_t> shape;  // extents, -1 for any; none given (rank -1): any shape
    int rank = -1;
    const c10::Device* device = nullptr;
    bool holds = true;
    std::string says;

    static Rule tensor(const Tensor& t, Elems e, std::vector<int64_t> shape, std::string says,
                       const c10::Device* dev = nullptr) {
        Rule r;
        r.t = &t;
        r.elems = e;
        r.rank = shape.empty() ? -1 : static_cast<int>(shape.size());  // no extents given: any shape
        r.shape = std::move(shape);
        r.device = dev;
        r.says = std::move(says);
        return r;
    }
    static Rule when(bool holds, std::string says) {
        Rule r;
        r.holds = holds;
        r.says = std::move(says);
        return r;
    }
};

bool rule_holds(const Rule& r) {
    if (r.t == nullptr) return r.holds;
    const Tensor& t = *r.t;
    if (r.device && t.device() != *r.device) return false;
    if (!elems_ok(t, r.elems)) return false;
    if (r.rank >= 0) {
        if (t.dim() != r.rank) return false;
        for (int i = 0; i < r.rank; ++i)
            if (r.shape[i] >= 0 && t.size(i) != r.shape[i]) return false;
    }
    return true;
}

// Checks the rules in order; the first that fails raises ValueError.
void enforce(std::initializer_list<Rule> rules) {
    for (const Rule& r : rules) TORCH_CHECK_VALUE(rule_holds(r), r.says);
}

// Engine status -> exception: ValueError for argument errors, RuntimeError otherwise.
void check_status(int status, const char* what) {
    TORCH_CHECK_VALUE(status != DBS_CUDA_STATUS_INVALID_ARGUMENT, "beamgrad CUDA ", what, ": invalid argument");
    TORCH_CHECK(status == DBS_CUDA_STATUS_OK, "beamgrad CUDA ", what, " failed: ", dbs_cuda_status_string(status));
}

std::string str(int64_t v) { return std::to_string(v); }

int dtype_code(const Tensor& t) {
    switch (t.scalar_type()) {
        case torch::kFloat16: return DBS_CUDA_DTYPE_F16;
        case torch::kBFloat16: return DBS_CUDA_DTYPE_BF16;
        default: return DBS_CUDA_DTYPE_F32;
    }
}

std::string dtype_message(const char* what, const Tensor& t) {
    return std::string(what) + " must be float32, float16 or bfloat16, got " + std::string(c10::toString(t.scalar_type()));
}

// Rules on the problem's sizes and search settings shared by the operators.
void enforce_problem(int64_t B, int64_t T, int64_t K, int64_t V, int64_t eos, int64_t min_length, double alpha,
                     double repetition) {
    auto extent = [](int64_t n, const char* name) {
        return Rule::when(n >= 1 && n <= kIntMax, std::string(name) + " must be in [1, INT_MAX], got " + str(n));
    };
    enforce({
        Rule::when(std::isfinite(alpha) && alpha >= 0.0, "length_penalty_alpha must be finite and non-negative"),
        Rule::when(std::isfinite(repetition) && repetition > 0.0, "repetition_penalty must be finite and positive"),
        extent(B, "B"), extent(T, "T"), extent(K, "K"), extent(V, "V"),
        Rule::when(K <= DBS_CUDA_MAX_BEAM,
                   "beam_size " + str(K) + " exceeds the CUDA backend maximum of " + str(DBS_CUDA_MAX_BEAM)),
        Rule::when(eos >= -1 && eos < V, "eos_token must be -1 or a token id < " + str(V)),
        Rule::when(min_length >= 0 && min_length <= kIntMax, "min_length must be non-negative"),
    });
}

// ---------------------------------------------------------------------------
// Host read-back: device values to check, read in one copy after the engine call
// ---------------------------------------------------------------------------
class HostCheck {
  public:
    // Queues `values` (read as int32) and a check run on them once read.
    void add(const Tensor& values, std::function<void(const int32_t*, int64_t)> check) {
        parts_.push_back(values.reshape({-1}).to(torch::kInt32));
        checks_.push_back(std::move(check));
    }
    bool empty() const { return parts_.empty(); }
    // One device-to-host copy (synchronizes the stream), then every check in order.
    void run() {
        if (parts_.empty()) return;
        const Tensor host = torch::cat(parts_).cpu();
        const int32_t* p = host.data_ptr<int32_t>();
        for (size_t i = 0; i < parts_.size(); ++i) {
            const int64_t n = parts_[i].numel();
            checks_[i](p, n);
            p += n;
        }
        parts_.clear();
        checks_.clear();
    }

  private:
    std::vector<Tensor> parts_;
    std::vector<std::function<void(const int32_t*, int64_t)>> checks_;
};

// Per-example step counts: an integer [B] tensor whose entries lie in [1, T]. The values are
// read back (one copy) and checked before the engine sees them; returned as int32 on `dev`.
OptTensor device_steps(const OptTensor& steps, const c10::Device& dev, int64_t B, int64_t T) {
    if (!steps.has_value()) return c10::nullopt;
    enforce({Rule::when(steps->dim() == 1 && steps->size(0) == B, "steps must have shape [B] = [" + str(B) + "]"),
             Rule::tensor(*steps, Elems::AnyInt, {-1}, "steps must be an integer tensor, got " +
                                                           std::string(c10::toString(steps->scalar_type())))});
    const Tensor wide = steps->to(torch::kInt64);
    const Tensor host = wide.cpu();
    const int64_t* v = host.data_ptr<int64_t>();
    for (int64_t b = 0; b < B; ++b)
        TORCH_CHECK_VALUE(v[b] >= 1 && v[b] <= T, "steps[", b, "] = ", v[b], " must be in [1, ", T, "]");
    return wide.to(dev, torch::kInt32).contiguous();
}

// The NaN/+inf flags of a validated decode, read with the other host checks.
void queue_flags(HostCheck& hc, const Tensor& invalid, std::string what) {
    hc.add(invalid, [what = std::move(what)](const int32_t* f, int64_t n) {
        for (int64_t b = 0; b < n; ++b)
            TORCH_CHECK_VALUE(f[b] == 0, "example ", b, ": ", what, " NaN or +inf in a row the search reads");
    });
}

// ---------------------------------------------------------------------------
// Problem description and search options for the engine
// ---------------------------------------------------------------------------
struct Problem {
    DBSCudaDecodeArgs args{};
    DBSCudaSearchOptions options{};
    Tensor steps, banned;  // device copies the args point into

    Problem(int64_t B, int64_t T, int64_t K, int64_t V, int64_t eos, int64_t min_length, double alpha,
            const OptTensor& steps_i32) {
        args.batch_size = static_cast<int>(B);
        args.steps = static_cast<int>(T);
        args.beam_size = static_cast<int>(K);
        args.vocab_size = static_cast<int>(V);
        args.eos_token = static_cast<int>(eos);
        args.min_length = static_cast<int>(min_length);
        args.length_penalty_alpha = static_cast<float>(alpha);
        args.repetition_penalty = 1.0f;
        if (steps_i32.has_value()) {
            steps = *steps_i32;
            args.steps_per_example = steps.data_ptr<int32_t>();
        }
    }

    void constrain(const OptTensor& banned_tokens, int64_t ngram, double repetition, const c10::Device& dev) {
        args.no_repeat_ngram_size = static_cast<int>(ngram < 0 ? 0 : (ngram > kIntMax ? kIntMax : ngram));
        args.repetition_penalty = static_cast<float>(repetition);
        if (!banned_tokens.has_value()) return;
        banned = banned_tokens->to(dev, torch::kUInt8).contiguous();
        enforce({Rule::when(banned.dim() == 1 && banned.size(0) == args.vocab_size, "banned_tokens must be a [V] mask")});
        args.banned_tokens = banned.data_ptr<uint8_t>();
    }

    void extra_eos(c10::IntArrayRef tokens) {
        const int64_t n = static_cast<int64_t>(tokens.size());
        enforce({Rule::when(n <= DBS_CUDA_MAX_EXTRA_EOS, "at most " + str(DBS_CUDA_MAX_EXTRA_EOS) +
                                                             " extra EOS tokens are supported on CUDA, got " + str(n)),
                 Rule::when(n == 0 || args.eos_token >= 0, "extra EOS tokens need eos_token >= 0")});
        for (int64_t tok : tokens) {
            enforce({Rule::when(tok >= 0 && tok < args.vocab_size, "extra EOS token " + str(tok) +
                                                                         " is outside the vocabulary (size " +
                                                                         str(args.vocab_size) + ")")});
            options.extra_eos_tokens[options.extra_eos_count++] = static_cast<int32_t>(tok);
        }
    }
};

// Engine workspace of `bytes` bytes (a negative size: the problem is outside the engine's limits).
Tensor workspace(int64_t bytes, const Tensor& like) {
    enforce({Rule::when(bytes >= 0,
                        "beamgrad CUDA: unsupported problem size (see DBS_CUDA_MAX_BEAM and the limits in dbs_cuda.h)")});
    return torch::empty({bytes > 0 ? bytes : 1}, like.options().dtype(torch::kUInt8));
}

// ---------------------------------------------------------------------------
// Output table: the trace tensors of a decode and the engine's pointers to them
// ---------------------------------------------------------------------------
enum Slot { kFinal, kFinalRaw, kFinalLen, kTokens, kParents, kLengths, kScores, kRaw, kFromLp, kRowLse, kInvalid,
            kSlots };

struct SlotSpec {
    bool per_step;             // [B, T, K] (else [B, K]; kInvalid: [B])
    c10::ScalarType type;
};
constexpr SlotSpec kSlotSpec[kSlots] = {
    {false, torch::kFloat32}, {false, torch::kFloat32}, {false, torch::kInt32}, {true, torch::kInt32},
    {true, torch::kInt32},    {true, torch::kInt32},    {true, torch::kFloat32}, {true, torch::kFloat32},
    {true, torch::kUInt8},    {true, torch::kFloat32},  {false, torch::kUInt8},
};

struct TraceOut {
    Tensor t[kSlots];
    DBSCudaDecodeOutputs view{};

    // Allocates the slots in `wanted` for a [B, T, K] decode on the device of `like`.
    TraceOut(const Tensor& like, int64_t B, int64_t T, int64_t K, const std::vector<Slot>& wanted) {
        for (Slot s : wanted) {
            const auto opts = like.options().dtype(kSlotSpec[s].type);
            t[s] = s == kInvalid ? torch::empty({B}, opts)
                                 : (kSlotSpec[s].per_step ? torch::empty({B, T, K}, opts) : torch::empty({B, K}, opts));
        }
        view.final_scores = ptr<float>(kFinal);
        view.final_raw_scores = ptr<float>(kFinalRaw);
        view.final_lengths = ptr<int32_t>(kFinalLen);
        view.tokens = ptr<int32_t>(kTokens);
        view.parents = ptr<int32_t>(kParents);
        view.lengths = ptr<int32_t>(kLengths);
        view.scores = ptr<float>(kScores);
        view.raw_scores = ptr<float>(kRaw);
        view.from_logprob = ptr<uint8_t>(kFromLp);
        view.invalid_input = ptr<uint8_t>(kInvalid);
    }
    template <class T>
    T* ptr(Slot s) {
        return t[s].defined() ? t[s].data_ptr<T>() : nullptr;
    }
};

using DecodeExResult = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;
using DecodeResult = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;
using StepResult = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;

// ---------------------------------------------------------------------------
// decode_ex / decode
// ---------------------------------------------------------------------------
DecodeExResult op_decode_ex(const Tensor& inputs, bool from_logits, const OptTensor& steps, int64_t eos_token,
                            int64_t min_length, double length_penalty_alpha, const OptTensor& banned_tokens,
                            int64_t no_repeat_ngram_size, double repetition_penalty, bool validate,
                            c10::IntArrayRef extra_eos) {
    TORCH_CHECK(inputs.is_cuda(), "beamgrad::decode (CUDA) expects a CUDA tensor");
    const char* what = from_logits ? "logits" : "log_probs";
    enforce({Rule::tensor(inputs, Elems::AnyFloat, {}, dtype_message(what, inputs)),
             Rule::when(inputs.dim() == 4, "inputs must have shape [B, T, K, V]")});
    const c10::cuda::CUDAGuard guard(inputs.device());
    const Tensor x = inputs.contiguous();
    const int64_t B = x.size(0), T = x.size(1), K = x.size(2), V = x.size(3);
    enforce_problem(B, T, K, V, eos_token, min_length, length_penalty_alpha, repetition_penalty);
    Problem pr(B, T, K, V, eos_token, min_length, length_penalty_alpha, device_steps(steps, x.device(), B, T));
    pr.constrain(banned_tokens, no_repeat_ngram_size, repetition_penalty, x.device());
    pr.extra_eos(extra_eos);
    std::vector<Slot> slots{kFinal, kFinalRaw, kFinalLen, kTokens, kParents, kLengths, kScores, kRaw, kFromLp, kRowLse};
    if (validate) slots.push_back(kInvalid);
    TraceOut out(x, B, T, K, slots);
    const int64_t ws_bytes = dbs_cuda_decode_workspace_size(&pr.args);
    const Tensor ws = workspace(ws_bytes, x);
    check_status(dbs_cuda_decode_ex2(x.data_ptr(), dtype_code(x), from_logits ? 1 : 0, &pr.args, &pr.options, &out.view,
                                     out.ptr<float>(kRowLse), ws.data_ptr(), ws_bytes, stream()),
                 "decode");
    if (validate) {
        HostCheck hc;
        queue_flags(hc, out.t[kInvalid], from_logits ? "logits contain" : "log_probs contains");
        hc.run();
    }
    return {out.t[kFinal], out.t[kFinalRaw], out.t[kFinalLen], out.t[kTokens], out.t[kParents],
            out.t[kLengths], out.t[kScores], out.t[kRaw], out.t[kFromLp], out.t[kRowLse]};
}

DecodeResult op_decode(const Tensor& log_probs, const OptTensor& steps, int64_t eos_token, int64_t min_length,
                       double length_penalty_alpha, const OptTensor& banned_tokens, int64_t no_repeat_ngram_size,
                       double repetition_penalty, bool validate) {
    enforce({Rule::tensor(log_probs, Elems::F32, {}, "log_probs must be float32")});
    const DecodeExResult r = op_decode_ex(log_probs, false, steps, eos_token, min_length, length_penalty_alpha,
                                          banned_tokens, no_repeat_ngram_size, repetition_penalty, validate, {});
    return {std::get<0>(r), std::get<1>(r), std::get<2>(r), std::get<3>(r), std::get<4>(r),
            std::get<5>(r), std::get<6>(r), std::get<7>(r), std::get<8>(r)};
}

// ---------------------------------------------------------------------------
// decode_step: one step from a caller-owned beam state (left untouched; the advanced
// state is returned)
// ---------------------------------------------------------------------------
StepResult op_decode_step(const Tensor& log_probs, const Tensor& raw_scores, const Tensor& lengths,
                          const Tensor& finished, const Tensor& prefixes, int64_t eos_token, int64_t min_length,
                          double length_penalty_alpha, const OptTensor& banned_tokens, int64_t no_repeat_ngram_size,
                          double repetition_penalty, bool validate, c10::IntArrayRef extra_eos) {
    TORCH_CHECK(log_probs.is_cuda(), "beamgrad::decode_step (CUDA) expects CUDA tensors");
    enforce({Rule::tensor(log_probs, Elems::F32, {-1, -1, -1}, "log_probs must be a float32 [B, K, V] tensor")});
    const c10::cuda::CUDAGuard guard(log_probs.device());
    const Tensor x = log_probs.contiguous();
    const c10::Device dev = x.device();
    const int64_t B = x.size(0), K = x.size(1), V = x.size(2);
    enforce({
        Rule::when(raw_scores.device() == dev && lengths.device() == dev && finished.device() == dev &&
                       prefixes.device() == dev,
                   "the beam state must be on the device of log_probs"),
        Rule::tensor(raw_scores, Elems::F32, {B, K}, "raw_scores must be a float32 [B, K] tensor"),
        Rule::tensor(lengths, Elems::I32, {B, K}, "lengths must be an int32 [B, K] tensor"),
        Rule::tensor(finished, Elems::U8, {B, K}, "finished must be a uint8 [B, K] tensor"),
        Rule::tensor(prefixes, Elems::I32, {B, K, -1}, "prefixes must be an int32 [B, K, L] tensor"),
        Rule::when(prefixes.dim() != 3 || prefixes.size(2) <= kIntMax, "prefixes must be an int32 [B, K, L] tensor"),
    });
    enforce_problem(B, 1, K, V, eos_token, min_length, length_penalty_alpha, repetition_penalty);
    Problem pr(B, 1, K, V, eos_token, min_length, length_penalty_alpha, c10::nullopt);
    pr.constrain(banned_tokens, no_repeat_ngram_size, repetition_penalty, dev);
    pr.extra_eos(extra_eos);

    // The engine advances the state it is given: it gets copies.
    Tensor next_raw = raw_scores.contiguous().clone();
    Tensor next_len = lengths.contiguous().clone();
    Tensor next_fin = finished.contiguous().clone();
    const Tensor pre = prefixes.contiguous();
    std::vector<Slot> slots{kFinal, kTokens, kParents, kScores, kFromLp};
    if (validate) slots.push_back(kInvalid);
    TraceOut out(x, B, 1, K, slots);
    DBSCudaBeamState state{};
    state.raw_scores = next_raw.data_ptr<float>();
    state.lengths = next_len.data_ptr<int32_t>();
    state.finished = next_fin.data_ptr<uint8_t>();
    state.prefixes = pre.numel() > 0 ? pre.data_ptr<int32_t>() : nullptr;
    state.prefix_stride = static_cast<int>(pre.size(2));

    HostCheck hc;
    if (validate && length_penalty_alpha != 0.0) {
        // The engine ranks a step's candidates by raw score, which is the CPU decoder's ranking
        // by penalised score when an example's live, unfinished beams share one length (true
        // of every state a search produces). Checked on the state as given.
        Tensor live = torch::isfinite(raw_scores);
        if (eos_token >= 0) live = live.logical_and(finished.eq(0));
        const Tensor shortest = torch::where(live, lengths, torch::full_like(lengths, kIntMax)).amin(1);
        const Tensor longest = torch::where(live, lengths, torch::full_like(lengths, -1)).amax(1);
        hc.add(torch::stack({shortest, longest}, 1), [](const int32_t* v, int64_t n) {
            for (int64_t b = 0; b < n / 2; ++b)
                TORCH_CHECK_VALUE(v[2 * b + 1] <= v[2 * b], "example ", b,
                                  ": with length_penalty_alpha != 0, decode_step on CUDA needs every live, unfinished "
                                  "beam to have the same length (as in any state the search produced), got lengths "
                                  "from ", v[2 * b], " to ", v[2 * b + 1]);
        });
    }
    const int64_t ws_bytes = dbs_cuda_decode_step_workspace_size(&pr.args, state.prefix_stride);
    const Tensor ws = workspace(ws_bytes, x);
    check_status(dbs_cuda_decode_step_ex2(x.data_ptr<float>(), DBS_CUDA_DTYPE_F32, 0, &pr.args, &pr.options, &state,
                                          &out.view, nullptr, ws.data_ptr(), ws_bytes, stream()),
                 "decode_step");
    if (validate) {
        queue_flags(hc, out.t[kInvalid], "log_probs contains");
        hc.run();
    }
    auto step = [](const Tensor& t) { return t.reshape({t.size(0), t.size(2)}); };  // [B, 1, K] -> [B, K]
    return {step(out.t[kTokens]), step(out.t[kParents]), next_len, step(out.t[kScores]), next_raw,
            step(out.t[kFromLp]), next_fin, out.t[kFinal]};
}

// ---------------------------------------------------------------------------
// Backward operators
// ---------------------------------------------------------------------------

// The trace a backward operator is given, checked and made contiguous.
struct TraceIn {
    Tensor parents, tokens, lengths, from_logprob;
    int64_t B = 0, T = 0, K = 0;
    DBSCudaBackwardInputs in{};

    TraceIn(const Tensor& par, const Tensor& tok, const Tensor& len, const Tensor& flp, const char* op) {
        TORCH_CHECK(par.is_cuda(), "beamgrad::", op, " (CUDA) expects CUDA tensors");
        enforce({Rule::tensor(par, Elems::I32, {-1, -1, -1}, "parents must be an int32 [B, T, K] tensor")});
        B = par.size(0);
        T = par.size(1);
        K = par.size(2);
        const c10::Device dev = par.device();
        enforce({
            Rule::tensor(tok, Elems::I32, {B, T, K}, "tokens and lengths must be int32 [B, T, K] tensors on the same device", &dev),
            Rule::tensor(len, Elems::I32, {B, T, K}, "tokens and lengths must be int32 [B, T, K] tensors on the same device", &dev),
            Rule::tensor(flp, Elems::U8, {B, T, K}, "from_logprob must be a uint8 [B, T, K] tensor on the same device", &dev),
        });
        parents = par.contiguous();
        tokens = tok.contiguous();
        lengths = len.contiguous();
        from_logprob = flp.contiguous();
        in.parents = parents.data_ptr<int32_t>();
        in.tokens = tokens.data_ptr<int32_t>();
        in.lengths = lengths.data_ptr<int32_t>();
        in.from_logprob = from_logprob.data_ptr<uint8_t>();
    }
    c10::Device device() const { return parents.device(); }

    // The decode's problem (its vocabulary, penalty and per-example steps) for the engine.
    Problem problem(int64_t V, double alpha, const OptTensor& steps) const {
        enforce_problem(B, T, K, V, -1, 0, alpha, 1.0);
        return Problem(B, T, K, V, -1, 0, alpha, device_steps(steps, device(), B, T));
    }
};

// An optional float32 gradient of `shape` on the trace's device: its pointer (null when
// absent); `keep` holds the contiguous copy.
const float* grad_input(const OptTensor& g, std::vector<int64_t> shape, const TraceIn& tr, const char* name, Tensor& keep) {
    if (!g.has_value()) return nullptr;
    const c10::Device dev = tr.device();
    std::string says = std::string(name) + " must be a float32 [";
    for (size_t i = 0; i < shape.size(); ++i) says += (i ? ", " : "") + str(shape[i]);
    says += "] tensor on the device of the trace";
    enforce({Rule::tensor(*g, Elems::F32, std::move(shape), says, &dev)});
    keep = g->contiguous();
    return keep.data_ptr<float>();
}

// The dense input gradient [B, T, K, V] in `out_type`, written once by dbs_cuda_backward_dense:
// equal to zero-filling a float32 gradient, accumulating the backward into it and casting the
// result to out_type.
Tensor dense_gradient(TraceIn& tr, Problem& pr, c10::ScalarType out_type) {
    int code = DBS_CUDA_DTYPE_F32;
    if (out_type == torch::kFloat16) code = DBS_CUDA_DTYPE_F16;
    else if (out_type == torch::kBFloat16) code = DBS_CUDA_DTYPE_BF16;
    else enforce({Rule::when(out_type == torch::kFloat32, "the gradient dtype must be float32, float16 or bfloat16")});
    Tensor grad = torch::empty({tr.B, tr.T, tr.K, pr.args.vocab_size}, tr.parents.options().dtype(out_type));
    const int64_t ws_bytes = dbs_cuda_backward_workspace_size(&pr.args);
    const Tensor ws = workspace(ws_bytes, tr.parents);
    check_status(dbs_cuda_backward_dense(&pr.args, &tr.in, grad.data_ptr(), code, ws.data_ptr(), ws_bytes, stream()),
                 "backward");
    return grad;
}

Tensor op_final_scores_backward(const Tensor& grad_final, const Tensor& parents, const Tensor& tokens,
                                const Tensor& lengths, const Tensor& from_logprob, const OptTensor& steps,
                                int64_t vocab_size, double length_penalty_alpha) {
    TraceIn tr(parents, tokens, lengths, from_logprob, "final_scores_backward");
    const c10::cuda::CUDAGuard guard(tr.device());
    Tensor g;
    tr.in.grad_final_scores = grad_input(grad_final, {tr.B, tr.K}, tr, "grad_final", g);
    Problem pr = tr.problem(vocab_size, length_penalty_alpha, steps);
    return dense_gradient(tr, pr, torch::kFloat32);
}

Tensor op_final_scores_path_gradient(const Tensor& grad_final, const Tensor& parents, const Tensor& tokens,
                                     const Tensor& lengths, const Tensor& from_logprob, const OptTensor& steps,
                                     int64_t vocab_size, double length_penalty_alpha) {
    TraceIn tr(parents, tokens, lengths, from_logprob, "final_scores_path_gradient");
    const c10::cuda::CUDAGuard guard(tr.device());
    Tensor g;
    const float* gp = grad_input(grad_final, {tr.B, tr.K}, tr, "grad_final", g);
    Problem pr = tr.problem(vocab_size, length_penalty_alpha, steps);
    Tensor draws = torch::empty({tr.B, tr.T, tr.K}, g.options());
    check_status(dbs_cuda_path_gradient(&pr.args, tr.in.parents, tr.in.tokens, tr.in.lengths, tr.in.from_logprob, gp,
                                        draws.data_ptr<float>(), stream()),
                 "path gradient");
    return draws;
}

Tensor decode_backward_in(const OptTensor& grad_final_scores, const OptTensor& grad_final_raw_scores,
                          const OptTensor& grad_scores, const OptTensor& grad_raw_scores, const Tensor& parents,
                          const Tensor& tokens, const Tensor& lengths, const Tensor& from_logprob,
                          const OptTensor& steps, int64_t vocab_size, double length_penalty_alpha,
                          const OptTensor& logits, const OptTensor& row_lse, c10::ScalarType out_type) {
    TraceIn tr(parents, tokens, lengths, from_logprob, "decode_backward");
    const c10::cuda::CUDAGuard guard(tr.device());
    Tensor keep[6];
    tr.in.grad_final_scores = grad_input(grad_final_scores, {tr.B, tr.K}, tr, "grad_final_scores", keep[0]);
    tr.in.grad_final_raw_scores = grad_input(grad_final_raw_scores, {tr.B, tr.K}, tr, "grad_final_raw_scores", keep[1]);
    tr.in.grad_scores = grad_input(grad_scores, {tr.B, tr.T, tr.K}, tr, "grad_scores", keep[2]);
    tr.in.grad_raw_scores = grad_input(grad_raw_scores, {tr.B, tr.T, tr.K}, tr, "grad_raw_scores", keep[3]);
    enforce({Rule::when(logits.has_value() == row_lse.has_value(), "logits and row_lse must be given together")});
    if (logits.has_value()) {
        const c10::Device dev = tr.device();
        enforce({
            Rule::tensor(*logits, Elems::AnyFloat, {}, dtype_message("logits", *logits)),
            Rule::tensor(*logits, Elems::AnyFloat, {tr.B, tr.T, tr.K, vocab_size},
                         "logits must be a [B, T, K, V] = [" + str(tr.B) + ", " + str(tr.T) + ", " + str(tr.K) + ", " +
                             str(vocab_size) + "] tensor on the same device",
                         &dev),
            Rule::tensor(*row_lse, Elems::F32, {tr.B, tr.T, tr.K},
                         "row_lse must be a float32 [B, T, K] tensor on the same device", &dev),
        });
        keep[4] = logits->contiguous();
        keep[5] = row_lse->contiguous();
        tr.in.logits = keep[4].data_ptr();
        tr.in.logits_type = dtype_code(keep[4]);
        tr.in.row_lse = keep[5].data_ptr<float>();
    }
    Problem pr = tr.problem(vocab_size, length_penalty_alpha, steps);
    return dense_gradient(tr, pr, out_type);
}

Tensor op_decode_backward(const OptTensor& grad_final_scores, const OptTensor& grad_final_raw_scores,
                          const OptTensor& grad_scores, const OptTensor& grad_raw_scores, const Tensor& parents,
                          const Tensor& tokens, const Tensor& lengths, const Tensor& from_logprob,
                          const OptTensor& steps, int64_t vocab_size, double length_penalty_alpha,
                          const OptTensor& logits, const OptTensor& row_lse) {
    return decode_backward_in(grad_final_scores, grad_final_raw_scores, grad_scores, grad_raw_scores, parents, tokens,
                              lengths, from_logprob, steps, vocab_size, length_penalty_alpha, logits, row_lse,
                              torch::kFloat32);
}

// beamgrad_b200::decode_backward_as: the gradient written directly in `dtype` (the input's
// dtype under autograd), in place of decode_backward(...).to(dtype) (python/beamgrad/
// _torch.py:289 of beamgrad 2.3.0).
Tensor op_decode_backward_as(const OptTensor& grad_final_scores, const OptTensor& grad_final_raw_scores,
                             const OptTensor& grad_scores, const OptTensor& grad_raw_scores, const Tensor& parents,
                             const Tensor& tokens, const Tensor& lengths, const Tensor& from_logprob,
                             const OptTensor& steps, int64_t vocab_size, double length_penalty_alpha,
                             const OptTensor& logits, const OptTensor& row_lse, c10::ScalarType dtype) {
    return decode_backward_in(grad_final_scores, grad_final_raw_scores, grad_scores, grad_raw_scores, parents, tokens,
                              lengths, from_logprob, steps, vocab_size, length_penalty_alpha, logits, row_lse, dtype);
}

Tensor op_length_penalty(const Tensor& lengths, double alpha) {
    TORCH_CHECK(lengths.is_cuda(), "beamgrad::length_penalty (CUDA) expects a CUDA tensor");
    enforce({Rule::tensor(lengths, Elems::AnyInt, {}, "lengths must be an integer tensor"),
             Rule::when(std::isfinite(alpha) && alpha >= 0.0, "length_penalty_alpha must be finite and non-negative")});
    const c10::cuda::CUDAGuard guard(lengths.device());
    const Tensor len = lengths.clamp(0, kIntMax).to(torch::kInt32).contiguous();
    Tensor out = torch::empty(len.sizes(), len.options().dtype(torch::kFloat32));
    check_status(dbs_cuda_length_penalty(len.data_ptr<int32_t>(), len.numel(), static_cast<float>(alpha),
                                         out.data_ptr<float>(), stream()),
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

// ---------------------------------------------------------------------------
// The Python module: device_available(), max_beam_size()
// ---------------------------------------------------------------------------
namespace {

PyObject* device_available(PyObject*, PyObject*) { return PyBool_FromLong(dbs_cuda_available() != 0); }
PyObject* max_beam_size(PyObject*, PyObject*) { return PyLong_FromLong(DBS_CUDA_MAX_BEAM); }

PyMethodDef kFunctions[] = {
    {"device_available", device_available, METH_NOARGS, "Whether the CUDA runtime reports a usable device"},
    {"max_beam_size", max_beam_size, METH_NOARGS, "Largest beam size the CUDA engine supports"},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef kModuleDef = {PyModuleDef_HEAD_INIT, "_C_cuda",
                          "CUDA kernels of the beamgrad operators (torch.ops.beamgrad.*) on the B200 engine", -1,
                          kFunctions};

}  // namespace

PyMODINIT_FUNC PyInit__C_cuda(void) { return PyModule_Create(&kModuleDef); }
