// torch_shim.cpp — host side of the drop-in boundary.
//
// Mirrors the reference's pybind11 bindings argument for argument, with the
// same validation messages and return layouts:
//   selective_scan_cuda.fwd_flat_ch / bwd_flat_ch
//       (csrc/selective_scan/selective_scan.cpp:674-1197)
//   extract_events_cuda.extract_base_events / expand_base_events /
//       gather_events_fwd / gather_events_bwd / extract_events
//       (csrc/extract/extract_events_cuda.cu:117-179, 324-798)
//   restore_dense_cuda_nodecay.restore_dense_fwd / restore_dense_bwd
//       (csrc/r_nodecay/restore_dense.cpp:41-226)
// Every device computation goes through the C ABI of libbcm_b200.so
// (include/bcm_b200.h); this file only validates, allocates with the ATen
// caching allocator and turns status codes into RuntimeError.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "bcm_b200.h"

#define CHECK_SHAPE(x, ...) \
    TORCH_CHECK(x.sizes() == torch::IntArrayRef({__VA_ARGS__}), #x " must have shape (" #__VA_ARGS__ ")")

namespace {

using at::Tensor;
using c10::optional;

// Error messages carry no integers formatted by TORCH_CHECK itself: with this
// torch build an integer in its message crashed the process instead of
// raising, so numbers go in as text.
void check_status(bcm_status st, const char* what) {
    if (st != BCM_OK) {
        const std::string code = std::to_string((int)st);
        TORCH_CHECK(false, what, ": ", bcm_last_error(), " (status ", code, ")");
    }
}

bcm_dtype to_bcm(at::ScalarType t, const char* what) {
    switch (t) {
        case at::ScalarType::Float: return BCM_F32;
        case at::ScalarType::Half: return BCM_F16;
        case at::ScalarType::BFloat16: return BCM_BF16;
        case at::ScalarType::Double: return BCM_F64;
        default: break;
    }
    TORCH_CHECK(false, what, " not implemented for type '", toString(t), "'");
    return BCM_F32;
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

Tensor workspace(int64_t bytes, const at::Device& dev) {
    return torch::empty({std::max<int64_t>(bytes, 1)},
                        torch::TensorOptions().dtype(torch::kUInt8).device(dev));
}

// ---------------------------------------------------------------- extract ----
// count pass (the given call) + fill, shared by both input layouts; the
// count call also brings the maximum per-channel count to the host (max_host)
// expand > 0: the fill writes the expanded stream directly (ch, ts, kf,
// expanded cu, max) instead of the base stream (ch, ts, kf, cu, counts, max),
// and with x_conv (B, D, L) also the gather of x_conv at it (sixth output)
template <typename CountFn>
std::vector<Tensor> extract_with(const Tensor& like, int64_t NCb, int64_t L, CountFn count, const char* what,
                                 int32_t* max_host = nullptr, int64_t expand = 0,
                                 const Tensor* x_conv = nullptr) {
    c10::cuda::CUDAGuard guard(like.device());
    auto opt_i = torch::TensorOptions().dtype(torch::kInt32).device(like.device());
    auto counts = torch::empty({NCb}, opt_i);
    auto cu = torch::empty({NCb + 1}, opt_i);
    auto mx = torch::empty({}, opt_i);
    auto ws = workspace((int64_t)bcm_extract_workspace_bytes(NCb, L), like.device());
    int64_t E = 0;
    int32_t mh = 0;
    check_status(count(counts, cu, mx, ws, &E, &mh), what);
    if (max_host) *max_host = mh;
    if (expand > 0) {
        TORCH_CHECK(E * expand < (1ll << 31) && NCb * expand < (1ll << 31), what, ": expanded sizes exceed int32");
        auto ch = torch::empty({E * expand}, opt_i);
        auto ts = torch::empty({E * expand}, opt_i);
        auto kf = torch::empty({E * expand}, opt_i);
        auto cu_x = torch::empty({NCb * expand + 1}, opt_i);
        Tensor x_flat;
        if (x_conv != nullptr) x_flat = torch::empty({E * expand}, x_conv->options());
        if (E == 0) {
            cu_x.zero_();
            if (x_conv != nullptr) return {ch, ts, kf, cu_x, torch::zeros({1}, opt_i), x_flat};
            return {ch, ts, kf, cu_x, torch::zeros({1}, opt_i)};
        }
        check_status(bcm_extract_expand_fill(NCb, L, cu.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(), expand,
                                             ch.data_ptr<int32_t>(), ts.data_ptr<int32_t>(),
                                             kf.data_ptr<int32_t>(), cu_x.data_ptr<int32_t>(),
                                             x_conv ? x_conv->data_ptr() : nullptr,
                                             x_conv ? to_bcm(x_conv->scalar_type(), what) : BCM_F32,
                                             x_conv ? x_flat.data_ptr() : nullptr, cur_stream()),
                     what);
        if (x_conv != nullptr) return {ch, ts, kf, cu_x, mx, x_flat};
        return {ch, ts, kf, cu_x, mx};
    }
    if (E == 0) {
        auto ei = torch::zeros({0}, opt_i);
        auto ms = torch::zeros({1}, opt_i);
        return {ei, ei, ei, cu, counts, ms};
    }
    auto ch = torch::empty({E}, opt_i);
    auto ts = torch::empty({E}, opt_i);
    auto kf = torch::empty({E}, opt_i);
    check_status(bcm_extract_base_fill(NCb, L, cu.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(),
                                       ch.data_ptr<int32_t>(), ts.data_ptr<int32_t>(),
                                       kf.data_ptr<int32_t>(), cur_stream()),
                 what);
    return {ch, ts, kf, cu, counts, mx};
}

std::vector<Tensor> extract_base_events_impl(const Tensor& base_input, double threshold, int32_t* max_host,
                                             int64_t expand = 0, const Tensor* x_conv = nullptr) {
    TORCH_CHECK(base_input.is_cuda(), "base_input must be CUDA");
    TORCH_CHECK(base_input.is_contiguous(), "base_input must be contiguous");
    TORCH_CHECK(base_input.dim() == 3, "base_input must be 3-D [B, d_model, L]");
    const bcm_dtype dt = to_bcm(base_input.scalar_type(), "count_base_kernel");
    const int64_t B = base_input.size(0), d_model = base_input.size(1), L = base_input.size(2);
    const float thr = (float)threshold;
    return extract_with(base_input, B * d_model, L,
                        [&](Tensor& counts, Tensor& cu, Tensor& mx, Tensor& ws, int64_t* E, int32_t* mh) {
                            return bcm_extract_base_count(base_input.data_ptr(), dt, B * d_model, L, thr,
                                                          counts.data_ptr<int32_t>(), cu.data_ptr<int32_t>(),
                                                          mx.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(), E,
                                                          mh, cur_stream());
                        },
                        "extract_base_events", max_host, expand, x_conv);
}

std::vector<Tensor> extract_base_events_fwd(Tensor base_input, double threshold) {
    return extract_base_events_impl(base_input, threshold, nullptr);
}

// Same outputs from the (B, L, d_model) layout (no transposed copy).
std::vector<Tensor> extract_base_events_bld_impl(const Tensor& x, double threshold, int32_t* max_host,
                                                 int64_t expand = 0, const Tensor* x_conv = nullptr) {
    TORCH_CHECK(x.is_cuda(), "x must be CUDA");
    TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
    TORCH_CHECK(x.dim() == 3, "x must be 3-D [B, L, d_model]");
    const bcm_dtype dt = to_bcm(x.scalar_type(), "extract_base_events_bld");
    const int64_t B = x.size(0), L = x.size(1), d_model = x.size(2);
    const float thr = (float)threshold;
    return extract_with(x, B * d_model, L,
                        [&](Tensor& counts, Tensor& cu, Tensor& mx, Tensor& ws, int64_t* E, int32_t* mh) {
                            return bcm_extract_base_count_bld(x.data_ptr(), dt, B, L, d_model, thr,
                                                              counts.data_ptr<int32_t>(), cu.data_ptr<int32_t>(),
                                                              mx.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(), E,
                                                              mh, cur_stream());
                        },
                        "extract_base_events_bld", max_host, expand, x_conv);
}

std::vector<Tensor> extract_base_events_bld_fwd(Tensor x, double threshold) {
    return extract_base_events_bld_impl(x, threshold, nullptr);
}

// The six outputs plus the maximum per-channel count as a host integer (read
// in the same synchronisation as the event total, so a caller that needs
// max_seqlen on the host makes no second synchronisation).
std::tuple<std::vector<Tensor>, int64_t> extract_base_events_host_max(Tensor base_input, double threshold,
                                                                       bool bld) {
    int32_t mh = 0;
    auto r = bld ? extract_base_events_bld_impl(base_input, threshold, &mh)
                 : extract_base_events_impl(base_input, threshold, &mh);
    return {r, (int64_t)mh};
}

// Extraction + expansion in one fill pass: the outputs of
// expand_base_events(*extract_base_events(x, threshold)[:4], B, d_model,
// expand) and the maximum per-channel count as a host integer (the one
// synchronisation of the count pass); bld selects the (B, L, d_model) layout.
// The first n elements of a larger buffer as a tensor of its own (same
// storage, no view relation to the buffer).
static Tensor head_of(const Tensor& buf, int64_t n) {
    Tensor t = at::empty({0}, buf.options());
    t.set_(buf.storage(), buf.storage_offset(), {n}, {1});
    return t;
}

// The fill of the expanded stream is enqueued before the host learns the
// event total, into capacity buffers whose first E*expand elements become the
// outputs (views: the whole capacity stays allocated while they live, e.g.
// saved for the backward).  The capacity is predicted per input shape from
// the largest totals of the last calls of that shape (kCapHeadroom above
// them), so a steady training loop pins little more than it uses; the first
// call of a shape, and any call whose total exceeds the prediction, fills
// after the synchronisation into exact-size outputs instead.  At most
// kAsyncFillBytes (BCM_ASYNC_FILL_BYTES overrides it) go to the capacity.
constexpr int64_t kAsyncFillBytes = int64_t(1) << 30;
constexpr double kCapHeadroom = 1.25;

struct CapKey {
    int dev;
    int64_t ncb, L, expand, xsize;
    bool operator<(const CapKey& o) const {
        return std::tie(dev, ncb, L, expand, xsize) < std::tie(o.dev, o.ncb, o.L, o.expand, o.xsize);
    }
};
struct CapHistory {
    int64_t recent[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int next = 0, seen = 0;
};
std::mutex g_cap_mu;
std::map<CapKey, CapHistory> g_cap;

// Predicted event total (expanded) of a call of this shape; 0 = no history.
int64_t predicted_events(const CapKey& k) {
    std::lock_guard<std::mutex> lock(g_cap_mu);
    auto it = g_cap.find(k);
    if (it == g_cap.end() || it->second.seen == 0) return 0;
    int64_t m = 0;
    for (int64_t v : it->second.recent) m = std::max(m, v);
    return (int64_t)(m * kCapHeadroom) + 4096;
}

void record_events(const CapKey& k, int64_t n) {
    std::lock_guard<std::mutex> lock(g_cap_mu);
    CapHistory& h = g_cap[k];
    h.recent[h.next] = n;
    h.next = (h.next + 1) % 8;
    h.seen += 1;
}

static int64_t async_fill_bytes() {
    const char* e = std::getenv("BCM_ASYNC_FILL_BYTES");
    return (e != nullptr && *e != '\0') ? std::max<int64_t>(0, std::atoll(e)) : kAsyncFillBytes;
}

std::tuple<std::vector<Tensor>, int64_t> extract_expanded_events(Tensor x, double threshold, int64_t expand,
                                                                  bool bld, const optional<Tensor>& x_conv,
                                                                  const optional<Tensor>& feature_thresholds,
                                                                  bool keep_mask) {
    const char* fn = "extract_expanded_events";
    TORCH_CHECK(expand >= 1, fn, ": expand must be >= 1");
    TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 3, fn, ": x must be a contiguous 3-D CUDA tensor");
    const int64_t B = x.size(0), L = bld ? x.size(1) : x.size(2), d_model = bld ? x.size(2) : x.size(1);
    const Tensor* xc = nullptr;
    if (x_conv.has_value() && x_conv->defined()) {
        const Tensor& v = *x_conv;
        TORCH_CHECK(v.is_cuda() && v.is_contiguous() && v.dim() == 3, fn,
                    ": x_conv must be a contiguous CUDA (B, D, L) tensor");
        TORCH_CHECK(v.device() == x.device(), fn, ": x_conv on x's device");
        TORCH_CHECK(v.size(0) == B && v.size(1) == d_model * expand && v.size(2) == L, fn,
                    ": x_conv must be (B, d_model*expand, L)");
        xc = &v;
    }
    const float* thr_ft = nullptr;
    if (feature_thresholds.has_value() && feature_thresholds->defined()) {
        const Tensor& t = *feature_thresholds;
        TORCH_CHECK(bld, fn, ": feature_thresholds need the (B, L, d_model) layout (bld=True)");
        TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous() && t.dim() == 1 &&
                        t.size(0) == d_model && t.device() == x.device(),
                    fn, ": feature_thresholds must be a contiguous float32 (d_model) tensor on x's device");
        thr_ft = t.data_ptr<float>();
    }
    const bcm_dtype dt = to_bcm(x.scalar_type(), fn);
    const int64_t NCb = B * d_model;
    TORCH_CHECK(NCb * expand < (1ll << 31), fn, ": expanded channels exceed int32");
    c10::cuda::CUDAGuard guard(x.device());
    auto opt_i = torch::TensorOptions().dtype(torch::kInt32).device(x.device());
    auto counts = torch::empty({NCb}, opt_i);
    auto base_cu = torch::empty({NCb + 1}, opt_i);
    auto mx = torch::empty({}, opt_i);
    auto ws = workspace((int64_t)bcm_extract_workspace_bytes(NCb, L), x.device());
    auto cu_x = torch::empty({NCb * expand + 1}, opt_i);
    // the fill runs before the host waits for the total, into buffers of the
    // predicted capacity; the outputs are their first E*expand elements
    const int64_t ub = std::min<int64_t>(NCb * L * expand, (1ll << 31) - 1);
    const int64_t per_event = 12 + (xc ? (int64_t)xc->element_size() : 0);
    const CapKey key{(int)x.device().index(), NCb, L, expand, xc ? (int64_t)xc->element_size() : 0};
    const int64_t cap = std::min<int64_t>({ub, async_fill_bytes() / per_event, predicted_events(key)});
    Tensor ch_c = torch::empty({cap}, opt_i), ts_c = torch::empty({cap}, opt_i), kf_c = torch::empty({cap}, opt_i);
    Tensor x_c;
    if (xc) x_c = torch::empty({cap}, xc->options());
    const bool fill_now = cap > 0;
    int64_t E = 0;
    int32_t mh = 0;
    int32_t* o_ch = fill_now ? ch_c.data_ptr<int32_t>() : nullptr;
    int32_t* o_ts = fill_now ? ts_c.data_ptr<int32_t>() : nullptr;
    int32_t* o_kf = fill_now ? kf_c.data_ptr<int32_t>() : nullptr;
    const void* g_x = (fill_now && xc) ? xc->data_ptr() : nullptr;
    const bcm_dtype g_dt = xc ? to_bcm(xc->scalar_type(), fn) : BCM_F32;
    void* g_out = (fill_now && xc) ? x_c.data_ptr() : nullptr;
    if (thr_ft) {
        check_status(bcm_extract_expanded_ft(x.data_ptr(), dt, B, d_model, L, thr_ft, expand,
                                             counts.data_ptr<int32_t>(), base_cu.data_ptr<int32_t>(),
                                             mx.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(), cap, o_ch, o_ts, o_kf,
                                             cu_x.data_ptr<int32_t>(), g_x, g_dt, g_out, &E, &mh, cur_stream()),
                     fn);
    } else {
        check_status(bcm_extract_expanded(x.data_ptr(), dt, bld ? 1 : 0, B, d_model, L, (float)threshold, expand,
                                          counts.data_ptr<int32_t>(), base_cu.data_ptr<int32_t>(),
                                          mx.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(), cap, o_ch, o_ts, o_kf,
                                          cu_x.data_ptr<int32_t>(), g_x, g_dt, g_out, &E, &mh, cur_stream()),
                     fn);
    }
    const int64_t n = E * expand;
    TORCH_CHECK(n < (1ll << 31), fn, ": expanded events exceed int32");
    record_events(key, n);
    Tensor ch, ts, kf, x_flat;
    if (n <= cap) {
        ch = head_of(ch_c, n);
        ts = head_of(ts_c, n);
        kf = head_of(kf_c, n);
        if (xc) x_flat = head_of(x_c, n);
    } else {
        ch = torch::empty({n}, opt_i);
        ts = torch::empty({n}, opt_i);
        kf = torch::empty({n}, opt_i);
        if (xc) x_flat = torch::empty({n}, xc->options());
        check_status(bcm_extract_expand_fill(NCb, L, base_cu.data_ptr<int32_t>(), ws.data_ptr(), ws.numel(), expand,
                                             ch.data_ptr<int32_t>(), ts.data_ptr<int32_t>(), kf.data_ptr<int32_t>(),
                                             cu_x.data_ptr<int32_t>(), xc ? xc->data_ptr() : nullptr,
                                             xc ? to_bcm(xc->scalar_type(), fn) : BCM_F32,
                                             xc ? x_flat.data_ptr() : nullptr, cur_stream()),
                     fn);
    }
    // expand_base_events' max is 0-d, or [0] of shape (1,) when nothing fires
    Tensor mo = (E == 0) ? torch::zeros({1}, opt_i) : mx;
    std::vector<Tensor> r = {ch, ts, kf, cu_x, mo};
    if (xc) r.push_back(x_flat);
    if (keep_mask) r.push_back(ws);   // its first words: the threshold mask [B*d_model][ceil(L/32)]
    return {r, (int64_t)mh};
}

std::vector<Tensor> expand_base_events_fwd(Tensor base_ch_ids, Tensor base_t_steps,
                                           Tensor base_k_flat, Tensor base_cu_seqlens,
                                           int64_t B, int64_t d_model, int64_t expand) {
    TORCH_CHECK(base_ch_ids.is_cuda(), "base_ch_ids must be CUDA");
    TORCH_CHECK(base_ch_ids.is_contiguous(), "base_ch_ids must be contiguous");
    c10::cuda::CUDAGuard guard(base_ch_ids.device());
    const int64_t NCb = B * d_model;
    const int64_t NCi = B * d_model * expand;
    const int64_t Eb = base_ch_ids.size(0);
    auto opt_i = torch::TensorOptions().dtype(torch::kInt32).device(base_ch_ids.device());
    if (Eb == 0) {
        auto cu = torch::zeros({NCi + 1}, opt_i);
        auto ms = torch::zeros({1}, opt_i);
        auto ei = torch::zeros({0}, opt_i);
        return {ei, ei, ei, cu, ms};
    }
    TORCH_CHECK(base_t_steps.is_contiguous() && base_k_flat.is_contiguous() &&
                    base_cu_seqlens.is_contiguous(),
                "expand_base_events: inputs must be contiguous");
    TORCH_CHECK(base_cu_seqlens.numel() >= NCb + 1,
                "expand_base_events: base_cu_seqlens must have B*d_model+1 entries");
    const int64_t E = Eb * expand;
    auto ch = torch::empty({E}, opt_i);
    auto ts = torch::empty({E}, opt_i);
    auto kf = torch::empty({E}, opt_i);
    auto cu = torch::empty({NCi + 1}, opt_i);
    auto mx = torch::empty({}, opt_i);
    check_status(bcm_expand_base_events(base_ch_ids.data_ptr<int32_t>(),
                                        base_t_steps.data_ptr<int32_t>(),
                                        base_k_flat.data_ptr<int32_t>(),
                                        base_cu_seqlens.data_ptr<int32_t>(), Eb, NCb, expand,
                                        ch.data_ptr<int32_t>(), ts.data_ptr<int32_t>(),
                                        kf.data_ptr<int32_t>(), cu.data_ptr<int32_t>(),
                                        mx.data_ptr<int32_t>(), cur_stream()),
                 "expand_base_events");
    return {ch, ts, kf, cu, mx};
}

std::vector<Tensor> gather_events_fwd(Tensor x, Tensor channel_ids, Tensor time_steps) {
    TORCH_CHECK(x.is_cuda(), "gather_events_fwd: x must be a CUDA tensor");
    TORCH_CHECK(x.is_contiguous(), "gather_events_fwd: x must be contiguous");
    TORCH_CHECK(channel_ids.scalar_type() == torch::kInt32, "gather_events_fwd: channel_ids must be int32");
    TORCH_CHECK(time_steps.scalar_type() == torch::kInt32, "gather_events_fwd: time_steps must be int32");
    TORCH_CHECK(x.dim() == 3, "gather_events_fwd: x must be 3-D [B, D, L]");
    c10::cuda::CUDAGuard guard(x.device());
    const int64_t L = x.size(2);
    const int64_t E = channel_ids.size(0);
    auto out = torch::empty({E}, x.options());
    if (E == 0) return {out};
    auto ch = channel_ids.contiguous();
    auto ts = time_steps.contiguous();
    check_status(bcm_gather_events_fwd(x.data_ptr(), to_bcm(x.scalar_type(), "gather_events_fwd"),
                                       x.size(0) * x.size(1), L, ch.data_ptr<int32_t>(),
                                       ts.data_ptr<int32_t>(), E, out.data_ptr(), cur_stream()),
                 "gather_events_fwd");
    return {out};
}

std::vector<Tensor> gather_events_bwd(Tensor grad_x, Tensor channel_ids, Tensor time_steps,
                                      int64_t NC, int64_t L) {
    TORCH_CHECK(grad_x.is_cuda(), "gather_events_bwd: grad tensor must be CUDA");
    TORCH_CHECK(channel_ids.scalar_type() == torch::kInt32, "gather_events_bwd: channel_ids must be int32");
    TORCH_CHECK(time_steps.scalar_type() == torch::kInt32, "gather_events_bwd: time_steps must be int32");
    c10::cuda::CUDAGuard guard(grad_x.device());
    auto g = grad_x.contiguous();
    auto dx = torch::empty({NC, L}, g.options());
    auto ch = channel_ids.contiguous();
    auto ts = time_steps.contiguous();
    Tensor ws = workspace((int64_t)bcm_gather_bwd_workspace_bytes(NC), g.device());
    check_status(bcm_gather_events_bwd(g.data_ptr(), to_bcm(g.scalar_type(), "gather_events_bwd"),
                                       ch.data_ptr<int32_t>(), ts.data_ptr<int32_t>(), g.size(0),
                                       NC, L, dx.data_ptr(), ws.data_ptr(), ws.numel(), cur_stream()),
                 "gather_events_bwd");
    return {dx};
}

// dx[NC, L] from a stream in extraction order and its cu_seqlens (no
// channel_ids pass): the gather autograd function's backward.
Tensor gather_events_bwd_rows(Tensor grad_x, Tensor time_steps, Tensor cu_seqlens, int64_t NC, int64_t L) {
    TORCH_CHECK(grad_x.is_cuda(), "gather_events_bwd_rows: grad tensor must be CUDA");
    TORCH_CHECK(time_steps.scalar_type() == torch::kInt32 && cu_seqlens.scalar_type() == torch::kInt32,
                "gather_events_bwd_rows: time_steps / cu_seqlens must be int32");
    TORCH_CHECK(cu_seqlens.numel() == NC + 1, "gather_events_bwd_rows: cu_seqlens must have NC + 1 entries");
    c10::cuda::CUDAGuard guard(grad_x.device());
    auto g = grad_x.contiguous();
    auto dx = torch::empty({NC, L}, g.options());
    auto ts = time_steps.contiguous();
    auto cu = cu_seqlens.contiguous();
    check_status(bcm_gather_events_bwd_rows(g.data_ptr(), to_bcm(g.scalar_type(), "gather_events_bwd_rows"),
                                            ts.data_ptr<int32_t>(), cu.data_ptr<int32_t>(), g.size(0), NC, L,
                                            dx.data_ptr(), nullptr, 0, cur_stream()),
                 "gather_events_bwd_rows");
    return dx;
}

static Tensor conv_weight2d(const Tensor& w, int64_t D);

// ------------------------------------------------------------------ decode
// One token of the event path for every channel; the state tensors are
// updated in place (eta [B*D, N] fp32, counters [B*D, 2] int32, held [B*D]
// fp32, conv_state [B, D, K] in x's dtype or None), y [B, D] is returned.
Tensor event_decode_step(Tensor x, Tensor spikes, double threshold, Tensor dt_idle, Tensor dt_active, Tensor A,
                         Tensor W_B, Tensor W_C, const optional<Tensor>& D_, Tensor eta, Tensor counters,
                         Tensor held, const optional<Tensor>& conv_state, const optional<Tensor>& conv_weight,
                         const optional<Tensor>& conv_bias) {
    const char* fn = "event_decode_step";
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), fn, ": x must be a contiguous CUDA (B, D) tensor");
    TORCH_CHECK(spikes.is_cuda() && spikes.dim() == 2 && spikes.is_contiguous() &&
                    spikes.scalar_type() == x.scalar_type() && spikes.size(0) == x.size(0),
                fn, ": spikes must be a contiguous (B, d_model) tensor of x's dtype");
    const int64_t B = x.size(0), D = x.size(1), dm = spikes.size(1), N = A.size(1);
    TORCH_CHECK(A.dim() == 2 && A.size(0) == D && A.scalar_type() == torch::kFloat32, fn, ": A must be fp32 (D, N)");
    auto f32 = [&](const Tensor& t, const char* name, std::vector<int64_t> shape) {
        TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous() && t.sizes() == shape,
                    fn, ": ", name, " has the wrong dtype, layout or shape");
    };
    f32(dt_idle, "dt_idle", {D}); f32(dt_active, "dt_active", {D});
    f32(W_B, "W_B", {D, N}); f32(W_C, "W_C", {D, N});
    f32(eta, "eta", {B * D, N}); f32(held, "held", {B * D});
    TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == torch::kInt32 && counters.is_contiguous() &&
                    counters.sizes() == torch::IntArrayRef({B * D, 2}),
                fn, ": counters must be int32 (B*D, 2)");
    const float* Dp = nullptr;
    if (D_.has_value() && D_->defined()) { f32(*D_, "D", {D}); Dp = D_->data_ptr<float>(); }
    void* cs = nullptr;
    const float* cw = nullptr;
    const float* cb = nullptr;
    int64_t K = 0;
    Tensor cw2;
    if (conv_state.has_value() && conv_state->defined()) {
        const Tensor& s = *conv_state;
        TORCH_CHECK(s.is_cuda() && s.is_contiguous() && s.dim() == 3 && s.size(0) == B && s.size(1) == D &&
                        s.scalar_type() == x.scalar_type(),
                    fn, ": conv_state must be a contiguous (B, D, K) tensor of x's dtype");
        TORCH_CHECK(conv_weight.has_value() && conv_weight->defined(), fn, ": conv_state needs conv_weight");
        K = s.size(2);
        cw2 = conv_weight2d(*conv_weight, D);
        TORCH_CHECK(cw2.size(1) == K, fn, ": conv_weight must have K taps");
        cs = s.data_ptr();
        cw = cw2.data_ptr<float>();
        if (conv_bias.has_value() && conv_bias->defined()) { f32(*conv_bias, "conv_bias", {D}); cb = conv_bias->data_ptr<float>(); }
    }
    c10::cuda::CUDAGuard guard(x.device());
    auto y = torch::empty_like(x);
    check_status(bcm_event_decode_step(x.data_ptr(), spikes.data_ptr(), to_bcm(x.scalar_type(), fn), B, D, dm, N,
                                       (float)threshold, dt_idle.data_ptr<float>(), dt_active.data_ptr<float>(),
                                       A.data_ptr<float>(), A.stride(0), A.stride(1), W_B.data_ptr<float>(),
                                       W_C.data_ptr<float>(), Dp, cs, cw, cb, K, eta.data_ptr<float>(),
                                       counters.data_ptr<int32_t>(), held.data_ptr<float>(), y.data_ptr(),
                                       cur_stream()),
                 fn);
    return y;
}

// ------------------------------------------------------------- conv at events
// weight [D, K] (or [D, 1, K]) and bias [D] are used as fp32.
static Tensor conv_weight2d(const Tensor& w, int64_t D) {
    TORCH_CHECK(w.is_cuda(), "conv_events: weight must be CUDA");
    Tensor w2 = w.dim() == 3 ? w.reshape({w.size(0), w.size(2)}) : w;
    TORCH_CHECK(w2.dim() == 2 && w2.size(0) == D, "conv_events: weight must be [D, K] or [D, 1, K]");
    return w2.to(torch::kFloat32).contiguous();
}

std::vector<Tensor> conv_events_fwd(Tensor x, Tensor weight, const optional<Tensor>& bias,
                                    Tensor channel_ids, Tensor time_steps) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 3, "conv_events_fwd: x must be a CUDA (B, D, L) tensor");
    TORCH_CHECK(channel_ids.scalar_type() == torch::kInt32 && time_steps.scalar_type() == torch::kInt32,
                "conv_events_fwd: channel_ids / time_steps must be int32");
    c10::cuda::CUDAGuard guard(x.device());
    auto xc = x.contiguous();
    const int64_t B = xc.size(0), D = xc.size(1), L = xc.size(2);
    auto w = conv_weight2d(weight, D);
    Tensor bv;
    if (bias.has_value() && bias->defined()) bv = bias->to(torch::kFloat32).contiguous();
    auto ch = channel_ids.contiguous();
    auto ts = time_steps.contiguous();
    auto out = torch::empty({ch.size(0)}, xc.options());
    check_status(bcm_conv_events_fwd(xc.data_ptr(), to_bcm(xc.scalar_type(), "conv_events_fwd"), B, D, L,
                                     w.data_ptr<float>(), bv.defined() ? bv.data_ptr<float>() : nullptr,
                                     w.size(1), ch.data_ptr<int32_t>(), ts.data_ptr<int32_t>(), ch.size(0),
                                     out.data_ptr(), cur_stream()),
                 "conv_events_fwd");
    return {out};
}

std::vector<Tensor> conv_events_bwd(Tensor x, Tensor weight, const optional<Tensor>& bias,
                                    Tensor time_steps, Tensor cu_seqlens, Tensor grad) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 3, "conv_events_bwd: x must be a CUDA (B, D, L) tensor");
    TORCH_CHECK(time_steps.scalar_type() == torch::kInt32 && cu_seqlens.scalar_type() == torch::kInt32,
                "conv_events_bwd: time_steps / cu_seqlens must be int32");
    c10::cuda::CUDAGuard guard(x.device());
    auto xc = x.contiguous();
    const int64_t B = xc.size(0), D = xc.size(1), L = xc.size(2);
    TORCH_CHECK(cu_seqlens.numel() == B * D + 1, "conv_events_bwd: cu_seqlens must have B*D+1 entries");
    auto w = conv_weight2d(weight, D);
    const int64_t K = w.size(1);
    Tensor bv;
    if (bias.has_value() && bias->defined()) bv = bias->to(torch::kFloat32).contiguous();
    auto g = grad.to(xc.scalar_type()).contiguous();
    auto ts = time_steps.contiguous();
    auto cu = cu_seqlens.contiguous();
    auto dx = torch::empty_like(xc);
    auto fopt = xc.options().dtype(torch::kFloat32);
    auto dw = torch::empty({D, K}, fopt);
    auto db = torch::empty({D}, fopt);
    Tensor ws = workspace((int64_t)bcm_conv_events_bwd_workspace_bytes(B * D, K), xc.device());
    check_status(bcm_conv_events_bwd(xc.data_ptr(), to_bcm(xc.scalar_type(), "conv_events_bwd"), B, D, L,
                                     w.data_ptr<float>(), bv.defined() ? bv.data_ptr<float>() : nullptr, K,
                                     ts.data_ptr<int32_t>(), cu.data_ptr<int32_t>(), ts.size(0), g.data_ptr(),
                                     dx.data_ptr(), dw.data_ptr<float>(), db.data_ptr<float>(), ws.data_ptr(),
                                     ws.numel(), cur_stream()),
                 "conv_events_bwd");
    return {dx, dw, db};
}

// Legacy bool-mask extraction (extract_events_cuda.cu:117-179): the same event
// stream as extract_base_events on mask > 0.5, plus head_flags.
std::vector<Tensor> extract_events_fwd(Tensor mask) {
    TORCH_CHECK(mask.is_cuda(), "mask must be a CUDA tensor");
    TORCH_CHECK(mask.is_contiguous(), "mask must be contiguous");
    TORCH_CHECK(mask.dtype() == torch::kBool, "mask must be bool");
    c10::cuda::CUDAGuard guard(mask.device());
    auto r = extract_base_events_fwd(mask.to(torch::kHalf), 0.5);
    auto ch = r[0], ts = r[1], kf = r[2], cu = r[3], counts = r[4];
    auto opt_i = torch::TensorOptions().dtype(torch::kInt32).device(mask.device());
    if (ch.numel() == 0) {
        auto ei = torch::zeros({0}, opt_i);
        return {ei, ei, ei, cu, torch::zeros({1}, opt_i), ei};
    }
    auto hflags = torch::zeros({ch.numel()}, opt_i);
    auto starts = cu.slice(0, 0, cu.numel() - 1).masked_select(counts > 0).to(torch::kLong);
    hflags.index_fill_(0, starts, 1);
    return {ch, ts, kf, cu, r[5], hflags};
}

// ------------------------------------------------------------------- scan ----
struct ScanPrep {
    bcm_flat_ch_args a{};
    Tensor u, k, cu, dti, dta, A, B, C, D, z, toff, pwB, pwC;
    bool depthwise = false, tiled = false, has_z = false, has_pw = false;
};

void prep_scan(ScanPrep& P, const char* fn, const Tensor& u_flat, const Tensor& k_flat,
               const Tensor& cu_seqlens, int64_t max_seqlen, const Tensor& dt_idle,
               const Tensor& dt_active, const Tensor& A, const Tensor& B, const Tensor& C,
               const optional<Tensor>& D_, const optional<Tensor>& z_,
               const optional<Tensor>& tile_offsets_, bool is_depthwise_bc,
               const optional<Tensor>& pw_B_, const optional<Tensor>& pw_C_, bool bwd) {
    const auto input_type = u_flat.scalar_type();
    TORCH_CHECK(input_type == at::ScalarType::Float || input_type == at::ScalarType::Half ||
                    input_type == at::ScalarType::BFloat16,
                fn, ": u_flat must be fp16/bf16/fp32");
    TORCH_CHECK(A.scalar_type() == at::ScalarType::Float, fn, ": A must be float32");
    TORCH_CHECK(B.scalar_type() == at::ScalarType::Float, fn, ": B must be float32");
    TORCH_CHECK(C.scalar_type() == at::ScalarType::Float, fn, ": C must be float32");
    TORCH_CHECK(u_flat.is_cuda() && k_flat.is_cuda() && cu_seqlens.is_cuda() && dt_idle.is_cuda() &&
                    dt_active.is_cuda() && A.is_cuda() && B.is_cuda() && C.is_cuda(),
                fn, ": all tensors must be CUDA tensors");
    TORCH_CHECK(u_flat.is_contiguous() && k_flat.is_contiguous() && cu_seqlens.is_contiguous(),
                fn, ": u_flat/k_flat/cu_seqlens must be contiguous");
    TORCH_CHECK(u_flat.dim() == 1, fn, ": u_flat must be 1-D");
    TORCH_CHECK(k_flat.dim() == 1, fn, ": k_flat must be 1-D");
    TORCH_CHECK(cu_seqlens.dim() == 1, fn, ": cu_seqlens must be 1-D");
    TORCH_CHECK(k_flat.scalar_type() == at::ScalarType::Int, fn, ": k_flat must be int32");
    TORCH_CHECK(cu_seqlens.scalar_type() == at::ScalarType::Int, fn, ": cu_seqlens must be int32");
    const int64_t E = u_flat.size(0);
    TORCH_CHECK(k_flat.size(0) == E, fn, ": k_flat must match u_flat shape");
    TORCH_CHECK(cu_seqlens.size(0) >= 2, fn, ": cu_seqlens must have at least 2 elements");
    const int64_t NC = cu_seqlens.size(0) - 1;
    TORCH_CHECK(dt_idle.scalar_type() == at::ScalarType::Float &&
                    dt_active.scalar_type() == at::ScalarType::Float,
                fn, ": dt_idle/dt_active must be float32");
    TORCH_CHECK(dt_idle.dim() == 1 && dt_active.dim() == 1, fn, ": dt_idle/dt_active must be 1-D");
    TORCH_CHECK(A.dim() == 2, fn, ": A must be 2-D (dim, dstate)");
    const int64_t dim = A.size(0), dstate = A.size(1);
    TORCH_CHECK(dstate <= 256, fn, ": dstate must be <= 256");
    CHECK_SHAPE(dt_idle, dim);
    CHECK_SHAPE(dt_active, dim);
    P.tiled = tile_offsets_.has_value() && tile_offsets_.value().defined();
    P.depthwise = is_depthwise_bc && !P.tiled;
    if (P.depthwise) {
        TORCH_CHECK(B.dim() == 2 && C.dim() == 2, fn, " (depthwise): W_B/W_C must be 2-D [dim, dstate]");
        TORCH_CHECK(B.size(0) == dim && B.size(1) == dstate, fn, " (depthwise): W_B must be [dim, dstate]");
        TORCH_CHECK(C.size(0) == dim && C.size(1) == dstate, fn, " (depthwise): W_C must be [dim, dstate]");
        TORCH_CHECK(B.is_contiguous() && C.is_contiguous(), fn, " (depthwise): W_B/W_C must be contiguous");
    } else if (P.tiled) {
        TORCH_CHECK(B.dim() == 3 && C.dim() == 3, fn,
                    ": tiled B/C must be 3-D [N_tiles, dstate, tile_chunk_size]");
        TORCH_CHECK(B.size(1) == dstate && C.size(1) == dstate, fn, ": tiled B/C dim-1 must equal dstate");
        TORCH_CHECK(B.is_contiguous() && C.is_contiguous(), fn, ": tiled B/C must be contiguous");
    } else if (!bwd) {
        TORCH_CHECK(B.dim() == 2 && C.dim() == 2, fn, ": B/C must be 2-D (dstate, E) [transposed layout]");
        CHECK_SHAPE(B, dstate, E);
        CHECK_SHAPE(C, dstate, E);
        TORCH_CHECK(B.stride(1) == 1 && C.stride(1) == 1, fn,
                    ": B/C must have contiguous last dimension (stride(1) == 1)");
    } else {
        TORCH_CHECK(B.dim() == 2 && C.dim() == 2, fn, ": B/C must be 2-D [dstate, E] or [dstate, dim]");
        TORCH_CHECK(B.stride(1) == 1 && C.stride(1) == 1, fn, ": B/C must have contiguous last dimension");
    }
    if (D_.has_value()) {
        TORCH_CHECK(D_.value().scalar_type() == at::ScalarType::Float, fn, ": D must be float32");
        TORCH_CHECK(D_.value().is_cuda() && D_.value().is_contiguous());
        CHECK_SHAPE(D_.value(), dim);
    }
    P.has_z = z_.has_value();
    if (P.has_z) {
        const Tensor& z = z_.value();
        TORCH_CHECK(z.scalar_type() == input_type, fn, ": z must have same dtype as u_flat");
        TORCH_CHECK(z.is_cuda() && z.is_contiguous());
        TORCH_CHECK(z.dim() == 1 && z.size(0) == E, fn, ": z must have shape (E,)");
    }
    TORCH_CHECK(max_seqlen >= 0, fn, ": max_seqlen must be non-negative");
    P.has_pw = P.depthwise && pw_B_.has_value() && pw_B_.value().defined();
    if (P.has_pw) {
        TORCH_CHECK(pw_C_.has_value() && pw_C_.value().defined(), fn, ": pw_C must accompany pw_B");
        const Tensor& pwB = pw_B_.value();
        const Tensor& pwC = pw_C_.value();
        TORCH_CHECK(pwB.scalar_type() == at::ScalarType::Float && pwC.scalar_type() == at::ScalarType::Float,
                    fn, ": pw_B/pw_C must be float32");
        TORCH_CHECK(pwB.is_cuda() && pwC.is_cuda() && pwB.is_contiguous() && pwC.is_contiguous(), fn,
                    ": pw_B/pw_C must be CUDA and contiguous");
        TORCH_CHECK(pwB.dim() == 2 && pwB.size(0) == dim && pwB.size(1) == dim, fn, ": pw_B must be [dim, dim]");
        TORCH_CHECK(pwC.dim() == 2 && pwC.size(0) == dim && pwC.size(1) == dim, fn, ": pw_C must be [dim, dim]");
        P.pwB = pwB;
        P.pwC = pwC;
    }
    P.u = u_flat; P.k = k_flat; P.cu = cu_seqlens;
    P.dti = dt_idle.contiguous(); P.dta = dt_active.contiguous();
    P.A = A;
    P.B = B.contiguous(); P.C = C.contiguous();
    if (D_.has_value()) P.D = D_.value();
    if (P.has_z) P.z = z_.value();
    if (P.tiled) P.toff = tile_offsets_.value().to(torch::kInt32).contiguous();

    bcm_flat_ch_args& a = P.a;
    a.n_events = E;
    a.n_channels = NC;
    a.dim = dim;
    a.dstate = dstate;
    a.max_seqlen = max_seqlen;
    a.dtype = to_bcm(input_type, fn);
    a.bc_mode = P.depthwise ? BCM_BC_DEPTHWISE : (P.tiled ? BCM_BC_TILED : BCM_BC_FLAT);
    a.b_variable = P.B.dim() == 2 ? (P.B.size(1) == E) : 1;
    a.c_variable = P.C.dim() == 2 ? (P.C.size(1) == E) : 1;
    a.u = P.u.data_ptr();
    a.k = P.k.data_ptr<int32_t>();
    a.cu_seqlens = P.cu.data_ptr<int32_t>();
    a.dt_idle = P.dti.data_ptr<float>();
    a.dt_active = P.dta.data_ptr<float>();
    a.A = P.A.data_ptr<float>();
    a.A_stride_d = P.A.stride(0);
    a.A_stride_n = P.A.stride(1);
    a.B = P.B.data_ptr<float>();
    a.C = P.C.data_ptr<float>();
    a.D = P.D.defined() ? P.D.data_ptr<float>() : nullptr;
    a.z = P.has_z ? P.z.data_ptr() : nullptr;
    a.tile_offsets = P.tiled ? P.toff.data_ptr<int32_t>() : nullptr;
    a.n_tiles = P.tiled ? std::min(P.B.size(0), P.C.size(0)) : 0;
    a.pw_B = P.has_pw ? P.pwB.data_ptr<float>() : nullptr;
    a.pw_C = P.has_pw ? P.pwC.data_ptr<float>() : nullptr;
}

// with_ckpt: the result gets one more entry, the state checkpoints for the
// backward (empty where the staged kernels do not run)
std::vector<Tensor> selective_scan_fwd_flat_ch_impl(
    const Tensor& u_flat, const Tensor& k_flat, const Tensor& cu_seqlens, const int64_t max_seqlen,
    const Tensor& dt_idle, const Tensor& dt_active, const Tensor& A, const Tensor& B,
    const Tensor& C, const optional<Tensor>& D_, const optional<Tensor>& z_,
    const optional<Tensor>& tile_offsets_, const int64_t tile_chunk_size, const bool is_depthwise_bc,
    const optional<Tensor>& pw_B_, const optional<Tensor>& pw_C_, bool with_ckpt) {
    (void)tile_chunk_size;  // the kernel derives the tile stride from max_seqlen, as the reference
    ScanPrep P;
    prep_scan(P, "selective_scan_fwd_flat_ch", u_flat, k_flat, cu_seqlens, max_seqlen, dt_idle,
              dt_active, A, B, C, D_, z_, tile_offsets_, is_depthwise_bc, pw_B_, pw_C_, false);
    c10::cuda::CUDAGuard guard(u_flat.device());
    int64_t n_chunks = (max_seqlen + 2047) / 2048;
    if (n_chunks == 0) n_chunks = 1;
    auto out = torch::empty_like(u_flat);
    auto x = torch::empty({P.a.n_channels, n_chunks, P.a.dstate * 2},
                          u_flat.options().dtype(torch::kFloat32));   // the forward writes every slot
    Tensor out_z;
    if (P.has_z) out_z = torch::empty_like(u_flat);
    bcm_flat_ch_args& a = P.a;
    a.out = out.data_ptr();
    a.x = x.data_ptr<float>();
    a.out_z = P.has_z ? out_z.data_ptr() : nullptr;
    Tensor ws = workspace((int64_t)bcm_flat_ch_fwd_workspace_bytes(&a), u_flat.device());
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws.numel();
    Tensor ckpt;
    if (with_ckpt) {
        const int64_t ck_bytes = (int64_t)bcm_flat_ch_ckpt_bytes(&a);
        ckpt = torch::empty({ck_bytes / 4}, u_flat.options().dtype(torch::kFloat32));
        a.ckpt = ck_bytes > 0 ? ckpt.data_ptr<float>() : nullptr;
    }
    check_status(bcm_flat_ch_fwd(&a, cur_stream()), "selective_scan_fwd_flat_ch");
    std::vector<Tensor> result = {out, x};
    if (P.has_z) result.push_back(out_z);
    if (with_ckpt) result.push_back(ckpt);
    return result;
}

std::vector<Tensor> selective_scan_fwd_flat_ch(
    const Tensor& u_flat, const Tensor& k_flat, const Tensor& cu_seqlens, const int64_t max_seqlen,
    const Tensor& dt_idle, const Tensor& dt_active, const Tensor& A, const Tensor& B,
    const Tensor& C, const optional<Tensor>& D_, const optional<Tensor>& z_,
    const optional<Tensor>& tile_offsets_, const int64_t tile_chunk_size, const bool is_depthwise_bc,
    const optional<Tensor>& pw_B_, const optional<Tensor>& pw_C_) {
    return selective_scan_fwd_flat_ch_impl(u_flat, k_flat, cu_seqlens, max_seqlen, dt_idle, dt_active, A, B, C,
                                           D_, z_, tile_offsets_, tile_chunk_size, is_depthwise_bc, pw_B_, pw_C_,
                                           false);
}

std::vector<Tensor> selective_scan_fwd_flat_ch_ckpt(
    const Tensor& u_flat, const Tensor& k_flat, const Tensor& cu_seqlens, const int64_t max_seqlen,
    const Tensor& dt_idle, const Tensor& dt_active, const Tensor& A, const Tensor& B,
    const Tensor& C, const optional<Tensor>& D_, const optional<Tensor>& z_,
    const optional<Tensor>& tile_offsets_, const int64_t tile_chunk_size, const bool is_depthwise_bc,
    const optional<Tensor>& pw_B_, const optional<Tensor>& pw_C_) {
    return selective_scan_fwd_flat_ch_impl(u_flat, k_flat, cu_seqlens, max_seqlen, dt_idle, dt_active, A, B, C,
                                           D_, z_, tile_offsets_, tile_chunk_size, is_depthwise_bc, pw_B_, pw_C_,
                                           true);
}

std::vector<Tensor> selective_scan_bwd_flat_ch(
    const Tensor& u_flat, const Tensor& k_flat, const Tensor& cu_seqlens, const int64_t max_seqlen,
    const Tensor& dt_idle, const Tensor& dt_active, const Tensor& A, const Tensor& B,
    const Tensor& C, const Tensor& dout_flat, const Tensor& x, const optional<Tensor>& D_,
    const optional<Tensor>& z_, const optional<Tensor>& out_, const optional<Tensor>& tile_offsets_,
    const int64_t tile_chunk_size, const bool is_depthwise_bc, const optional<Tensor>& pw_B_,
    const optional<Tensor>& pw_C_, const optional<Tensor>& ckpt_) {
    (void)tile_chunk_size;
    const char* fn = "selective_scan_bwd_flat_ch";
    TORCH_CHECK(dout_flat.scalar_type() == u_flat.scalar_type(), fn, ": dout_flat must match u_flat dtype");
    TORCH_CHECK(dout_flat.is_cuda() && x.is_cuda(), fn, ": all tensors must be CUDA tensors");
    TORCH_CHECK(dout_flat.is_contiguous(), fn, ": u_flat/k_flat/cu_seqlens/dout_flat must be contiguous");
    TORCH_CHECK(dout_flat.dim() == 1, fn, ": u_flat/k_flat/cu_seqlens/dout_flat must be 1-D");
    ScanPrep P;
    prep_scan(P, fn, u_flat, k_flat, cu_seqlens, max_seqlen, dt_idle, dt_active, A, B, C, D_, z_,
              tile_offsets_, is_depthwise_bc, pw_B_, pw_C_, true);
    TORCH_CHECK(dout_flat.size(0) == u_flat.size(0), fn, ": dout_flat must match u_flat shape");
    c10::cuda::CUDAGuard guard(u_flat.device());
    bcm_flat_ch_args& a = P.a;
    TORCH_CHECK(x.scalar_type() == at::ScalarType::Float, fn, ": x must be float32");
    TORCH_CHECK(x.is_contiguous(), fn, ": x must be contiguous");
    TORCH_CHECK(x.dim() == 3 && x.size(0) == a.n_channels && x.size(2) == a.dstate * 2, fn,
                ": x must have shape (n_channels, n_chunks, dstate*2)");
    int64_t n_chunks = (max_seqlen + 2047) / 2048;
    if (n_chunks == 0) n_chunks = 1;
    TORCH_CHECK(x.size(1) == n_chunks, fn, ": x.size(1) must equal n_chunks = (max_seqlen + 2047) / 2048");
    Tensor out_fwd, dz;
    if (P.has_z) {
        TORCH_CHECK(out_.has_value(), fn,
                    ": out (forward ungated output) must be provided when z is provided");
        out_fwd = out_.value();
        TORCH_CHECK(out_fwd.scalar_type() == u_flat.scalar_type(), fn, ": z/out must match u_flat dtype");
        TORCH_CHECK(out_fwd.is_cuda() && out_fwd.is_contiguous());
        TORCH_CHECK(out_fwd.size(0) == u_flat.size(0), fn, ": z/out must have shape (E,)");
        dz = torch::zeros_like(u_flat);
    }
    auto du = torch::empty_like(u_flat);
    auto dA = torch::empty_like(A, at::MemoryFormat::Contiguous);
    Tensor dB, dC;
    if (P.depthwise) {
        dB = torch::empty_like(P.B);
        dC = torch::empty_like(P.C);
    } else {
        dB = torch::zeros_like(P.B);
        dC = torch::zeros_like(P.C);
    }
    auto ddt_idle = torch::empty_like(dt_idle);
    auto ddt_active = torch::empty_like(dt_active);
    Tensor dD, dpwB, dpwC;
    if (D_.has_value()) dD = torch::empty_like(D_.value());
    if (P.has_pw) {
        dpwB = torch::empty_like(P.pwB);
        dpwC = torch::empty_like(P.pwC);
    }
    a.x = x.data_ptr<float>();
    a.dout = dout_flat.data_ptr();
    a.out_fwd = P.has_z ? out_fwd.data_ptr() : nullptr;
    a.du = du.data_ptr();
    a.dA = dA.data_ptr<float>();
    a.dB = dB.data_ptr<float>();
    a.dC = dC.data_ptr<float>();
    a.ddt_idle = ddt_idle.data_ptr<float>();
    a.ddt_active = ddt_active.data_ptr<float>();
    a.dD = dD.defined() ? dD.data_ptr<float>() : nullptr;
    a.dz = P.has_z ? dz.data_ptr() : nullptr;
    a.dpw_B = P.has_pw ? dpwB.data_ptr<float>() : nullptr;
    a.dpw_C = P.has_pw ? dpwC.data_ptr<float>() : nullptr;
    Tensor ws = workspace((int64_t)bcm_flat_ch_bwd_workspace_bytes(&a), u_flat.device());
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws.numel();
    if (ckpt_.has_value() && ckpt_->defined() && ckpt_->numel() > 0) {
        const Tensor& ck = *ckpt_;
        TORCH_CHECK(ck.is_cuda() && ck.scalar_type() == at::ScalarType::Float && ck.is_contiguous() &&
                        ck.numel() * 4 == (int64_t)bcm_flat_ch_ckpt_bytes(&a),
                    fn, ": ckpt must be the checkpoints fwd_flat_ch_ckpt returned for these inputs");
        a.ckpt = ck.data_ptr<float>();
    }
    check_status(bcm_flat_ch_bwd(&a, cur_stream()), fn);
    std::vector<Tensor> result = {du, dA, dB, dC, ddt_idle, ddt_active};
    if (D_.has_value()) result.push_back(dD);
    if (P.has_z) result.push_back(dz);
    if (P.has_pw) {
        result.push_back(dpwB);
        result.push_back(dpwC);
    }
    return result;
}

// ------------------------------------------------------------- dense S6 ----
// selective_scan_cuda.fwd / .bwd (reference csrc/selective_scan/selective_scan.cpp:
// 403-497 and 499-669): same arguments, checks, messages and outputs, real
// weights (complex A is rejected with a clear message).
struct S6In {
    bool varB, varC;
    int64_t batch, dim, L, N, groups;
    Tensor Bc, Cc;
};

S6In s6_check(const Tensor& u, const Tensor& delta, const Tensor& A, const Tensor& B, const Tensor& C,
              const optional<Tensor>& D_, const optional<Tensor>& delta_bias_) {
    auto input_type = u.scalar_type();
    auto weight_type = A.scalar_type();
    TORCH_CHECK(input_type == at::ScalarType::Float || input_type == at::ScalarType::Half ||
                input_type == at::ScalarType::BFloat16);
    TORCH_CHECK(weight_type == at::ScalarType::Float || weight_type == at::ScalarType::ComplexFloat);
    TORCH_CHECK(weight_type == at::ScalarType::Float,
                "selective_scan: complex weights are not supported by this build");
    S6In s;
    s.varB = B.dim() >= 3;
    s.varC = C.dim() >= 3;
    TORCH_CHECK(delta.scalar_type() == input_type);
    TORCH_CHECK(B.scalar_type() == (!s.varB ? weight_type : input_type));
    TORCH_CHECK(C.scalar_type() == (!s.varC ? weight_type : input_type));
    TORCH_CHECK(u.is_cuda());
    TORCH_CHECK(delta.is_cuda());
    TORCH_CHECK(A.is_cuda());
    TORCH_CHECK(B.is_cuda());
    TORCH_CHECK(C.is_cuda());
    TORCH_CHECK(u.stride(-1) == 1 || u.size(-1) == 1);
    TORCH_CHECK(delta.stride(-1) == 1 || delta.size(-1) == 1);
    TORCH_CHECK(u.dim() == 3, "u must have shape (batch, dim, seqlen)");
    s.batch = u.size(0);
    s.dim = u.size(1);
    s.L = u.size(2);
    s.N = A.size(1);
    s.groups = s.varB ? B.size(1) : 1;
    TORCH_CHECK(s.N <= 256, "selective_scan only supports state dimension <= 256");
    TORCH_CHECK(delta.sizes() == u.sizes(), "delta must have shape (batch, dim, seqlen)");
    TORCH_CHECK(A.dim() == 2 && A.size(0) == s.dim, "A must have shape (dim, dstate)");
    auto check_bc = [&](const Tensor& X, bool var, const char* name) {
        if (!var) {
            TORCH_CHECK(X.dim() == 2 && X.size(0) == s.dim && X.size(1) == s.N, name,
                        " must have shape (dim, dstate)");
        } else {
            TORCH_CHECK(X.dim() == 4 && X.size(0) == s.batch && X.size(1) == s.groups && X.size(2) == s.N &&
                            X.size(3) == s.L,
                        name, " must have shape (batch, n_groups, dstate, seqlen)");
            TORCH_CHECK(X.stride(-1) == 1 || X.size(-1) == 1);
        }
    };
    check_bc(B, s.varB, "B");
    check_bc(C, s.varC, "C");
    TORCH_CHECK(!(s.varB || s.varC) || s.dim % s.groups == 0, "dim must be a multiple of n_groups");
    if (D_.has_value()) {
        auto D = D_.value();
        TORCH_CHECK(D.scalar_type() == at::ScalarType::Float);
        TORCH_CHECK(D.is_cuda());
        TORCH_CHECK(D.stride(-1) == 1 || D.size(-1) == 1);
        TORCH_CHECK(D.dim() == 1 && D.size(0) == s.dim, "D must have shape (dim,)");
    }
    if (delta_bias_.has_value()) {
        auto delta_bias = delta_bias_.value();
        TORCH_CHECK(delta_bias.scalar_type() == at::ScalarType::Float);
        TORCH_CHECK(delta_bias.is_cuda());
        TORCH_CHECK(delta_bias.stride(-1) == 1 || delta_bias.size(-1) == 1);
        TORCH_CHECK(delta_bias.dim() == 1 && delta_bias.size(0) == s.dim, "delta_bias must have shape (dim,)");
    }
    s.Bc = s.varB ? B.contiguous() : B;
    s.Cc = s.varC ? C.contiguous() : C;
    return s;
}

bcm_s6_args s6_args(const S6In& s, const Tensor& u, const Tensor& delta, const Tensor& A,
                    const optional<Tensor>& D_, const optional<Tensor>& delta_bias_, bool delta_softplus) {
    bcm_s6_args a{};
    a.batch = s.batch; a.dim = s.dim; a.seqlen = s.L; a.dstate = s.N; a.n_groups = s.groups;
    a.dtype = to_bcm(u.scalar_type(), "selective_scan");
    a.is_variable_B = s.varB; a.is_variable_C = s.varC; a.delta_softplus = delta_softplus;
    a.u = u.data_ptr(); a.u_stride_b = u.stride(0); a.u_stride_d = u.stride(1);
    a.delta = delta.data_ptr(); a.delta_stride_b = delta.stride(0); a.delta_stride_d = delta.stride(1);
    a.A = A.data_ptr<float>(); a.A_stride_d = A.stride(0); a.A_stride_n = A.stride(1);
    a.B = s.Bc.data_ptr(); a.C = s.Cc.data_ptr();
    if (!s.varB) { a.B_stride_d = s.Bc.stride(0); a.B_stride_n = s.Bc.stride(1); }
    if (!s.varC) { a.C_stride_d = s.Cc.stride(0); a.C_stride_n = s.Cc.stride(1); }
    a.D = D_.has_value() ? D_.value().data_ptr<float>() : nullptr;
    a.delta_bias = delta_bias_.has_value() ? delta_bias_.value().data_ptr<float>() : nullptr;
    return a;
}

std::vector<Tensor> selective_scan_fwd(const Tensor& u, const Tensor& delta, const Tensor& A, const Tensor& B,
                                       const Tensor& C, const optional<Tensor>& D_, const optional<Tensor>& z_,
                                       const optional<Tensor>& delta_bias_, bool delta_softplus) {
    S6In s = s6_check(u, delta, A, B, C, D_, delta_bias_);
    Tensor z, out_z;
    const bool has_z = z_.has_value();
    if (has_z) {
        z = z_.value();
        TORCH_CHECK(z.scalar_type() == u.scalar_type());
        TORCH_CHECK(z.is_cuda());
        TORCH_CHECK(z.stride(-1) == 1 || z.size(-1) == 1);
        TORCH_CHECK(z.sizes() == u.sizes(), "z must have shape (batch, dim, seqlen)");
        z = z.contiguous();
        out_z = torch::empty(u.sizes(), z.options());
    }
    const int64_t n_chunks = (s.L + 2048 - 1) / 2048;
    Tensor out = torch::empty(u.sizes(), delta.options());
    Tensor x = torch::empty({s.batch, s.dim, n_chunks, s.N * 2}, u.options().dtype(A.scalar_type()));
    c10::cuda::CUDAGuard device_guard(u.device());
    bcm_s6_args a = s6_args(s, u, delta, A, D_, delta_bias_, delta_softplus);
    a.z = has_z ? z.data_ptr() : nullptr;
    a.out = out.data_ptr();
    a.out_z = has_z ? out_z.data_ptr() : nullptr;
    a.x = x.data_ptr<float>();
    check_status(bcm_s6_fwd(&a, cur_stream()), "selective_scan_fwd");
    std::vector<Tensor> result = {out, x};
    if (has_z) result.push_back(out_z);
    return result;
}

std::vector<Tensor> selective_scan_bwd(const Tensor& u, const Tensor& delta, const Tensor& A, const Tensor& B,
                                       const Tensor& C, const optional<Tensor>& D_, const optional<Tensor>& z_,
                                       const optional<Tensor>& delta_bias_, const Tensor& dout,
                                       const optional<Tensor>& x_, const optional<Tensor>& out_,
                                       optional<Tensor> dz_, bool delta_softplus, bool recompute_out_z) {
    S6In s = s6_check(u, delta, A, B, C, D_, delta_bias_);
    TORCH_CHECK(dout.scalar_type() == u.scalar_type());
    TORCH_CHECK(dout.is_cuda());
    TORCH_CHECK(dout.stride(-1) == 1 || dout.size(-1) == 1);
    TORCH_CHECK(dout.sizes() == u.sizes(), "dout must have shape (batch, dim, seqlen)");
    Tensor z, out, dz, out_z;
    const bool has_z = z_.has_value();
    if (has_z) {
        z = z_.value();
        TORCH_CHECK(z.scalar_type() == u.scalar_type());
        TORCH_CHECK(z.is_cuda());
        TORCH_CHECK(z.stride(-1) == 1 || z.size(-1) == 1);
        TORCH_CHECK(z.sizes() == u.sizes(), "z must have shape (batch, dim, seqlen)");
        TORCH_CHECK(out_.has_value());
        out = out_.value();
        TORCH_CHECK(out.scalar_type() == u.scalar_type());
        TORCH_CHECK(out.is_cuda());
        TORCH_CHECK(out.stride(-1) == 1 || out.size(-1) == 1);
        TORCH_CHECK(out.sizes() == u.sizes(), "out must have shape (batch, dim, seqlen)");
        z = z.contiguous();
        out = out.contiguous();
        if (dz_.has_value()) {
            dz = dz_.value();
            TORCH_CHECK(dz.scalar_type() == u.scalar_type());
            TORCH_CHECK(dz.is_cuda());
            TORCH_CHECK(dz.stride(-1) == 1 || dz.size(-1) == 1);
            TORCH_CHECK(dz.sizes() == u.sizes(), "dz must have shape (batch, dim, seqlen)");
            TORCH_CHECK(dz.is_contiguous(), "dz must be contiguous");
        } else {
            dz = torch::empty(u.sizes(), z.options());
        }
        if (recompute_out_z) out_z = torch::empty(u.sizes(), out.options());
    }
    const int64_t n_chunks = (s.L + 2048 - 1) / 2048;
    if (n_chunks > 1) { TORCH_CHECK(x_.has_value()); }
    if (x_.has_value()) {
        auto x = x_.value();
        TORCH_CHECK(x.scalar_type() == A.scalar_type());
        TORCH_CHECK(x.is_cuda());
        TORCH_CHECK(x.is_contiguous());
        TORCH_CHECK(x.dim() == 4 && x.size(0) == s.batch && x.size(1) == s.dim && x.size(2) == n_chunks &&
                        x.size(3) == 2 * s.N,
                    "x must have shape (batch, dim, n_chunks, 2 * dstate)");
    }
    Tensor doutc = dout.contiguous();
    Tensor du = torch::empty(u.sizes(), u.options());
    Tensor ddelta = torch::empty(u.sizes(), delta.options());
    Tensor dA = torch::zeros_like(A);
    Tensor dB = !s.varB ? torch::zeros_like(B) : torch::zeros_like(B, B.options().dtype(torch::kFloat32));
    Tensor dC = !s.varC ? torch::zeros_like(C) : torch::zeros_like(C, C.options().dtype(torch::kFloat32));
    Tensor dD, ddelta_bias;
    if (D_.has_value()) dD = torch::zeros_like(D_.value());
    if (delta_bias_.has_value()) ddelta_bias = torch::zeros_like(delta_bias_.value());
    TORCH_CHECK(dA.is_contiguous() && dB.is_contiguous() && dC.is_contiguous(),
                "selective_scan_bwd: A, B and C must be contiguous");
    c10::cuda::CUDAGuard device_guard(u.device());
    bcm_s6_args a = s6_args(s, u, delta, A, D_, delta_bias_, delta_softplus);
    a.z = has_z ? z.data_ptr() : nullptr;
    a.dout = doutc.data_ptr();
    a.out_fwd = has_z ? out.data_ptr() : nullptr;
    a.du = du.data_ptr();
    a.ddelta = ddelta.data_ptr();
    a.dA = dA.data_ptr<float>();
    a.dB = dB.data_ptr<float>();
    a.dC = dC.data_ptr<float>();
    a.dD = D_.has_value() ? dD.data_ptr<float>() : nullptr;
    a.ddelta_bias = delta_bias_.has_value() ? ddelta_bias.data_ptr<float>() : nullptr;
    a.dz = has_z ? dz.data_ptr() : nullptr;
    a.out_z = (has_z && recompute_out_z) ? out_z.data_ptr() : nullptr;
    Tensor ws = workspace((int64_t)bcm_s6_bwd_workspace_bytes(&a), u.device());
    a.workspace = ws.data_ptr();
    a.workspace_bytes = (size_t)ws.numel();
    check_status(bcm_s6_bwd(&a, cur_stream()), "selective_scan_bwd");
    std::vector<Tensor> result = {du, ddelta, dA, dB.to(B.dtype()), dC.to(C.dtype()), dD, ddelta_bias};
    if (has_z) result.push_back(dz);
    if (recompute_out_z) result.push_back(out_z);
    return result;
}

// ---------------------------------------------------------------- restore ----
// bitmap != nullptr: also returns the event bitmap words ([B, ceil(L/32), dim]) and the sweep's
// per-unit start indices, one flat int32 buffer for restore_dense_bwd_bitmap
Tensor restore_fwd_impl(const Tensor& y_flat, const Tensor& time_steps, const Tensor& cu_seqlens,
                        int64_t dim, int64_t seqlen, const optional<at::ScalarType> out_dtype_opt,
                        Tensor* bitmap, const Tensor* base_mask = nullptr, int64_t expand = 1) {
    auto input_type = y_flat.scalar_type();
    TORCH_CHECK(input_type == at::ScalarType::Float || input_type == at::ScalarType::Half ||
                    input_type == at::ScalarType::BFloat16,
                "restore_dense_fwd: y_flat must be fp32, fp16, or bf16");
    TORCH_CHECK(time_steps.scalar_type() == at::ScalarType::Int,
                "restore_dense_fwd: time_steps must be int32 (torch.int32)");
    TORCH_CHECK(cu_seqlens.scalar_type() == at::ScalarType::Int,
                "restore_dense_fwd: cu_seqlens must be int32 (torch.int32)");
    TORCH_CHECK(y_flat.is_cuda() && time_steps.is_cuda() && cu_seqlens.is_cuda(),
                "restore_dense_fwd: all tensors must be on CUDA");
    TORCH_CHECK(y_flat.is_contiguous() && time_steps.is_contiguous() && cu_seqlens.is_contiguous(),
                "restore_dense_fwd: all tensors must be contiguous");
    TORCH_CHECK(y_flat.dim() == 1, "restore_dense_fwd: y_flat must be 1-D");
    TORCH_CHECK(time_steps.sizes() == y_flat.sizes(), "restore_dense_fwd: time_steps shape must equal y_flat shape");
    TORCH_CHECK(cu_seqlens.dim() == 1, "restore_dense_fwd: cu_seqlens must be 1-D");
    TORCH_CHECK(dim >= 1, "restore_dense_fwd: dim must be >= 1");
    TORCH_CHECK(seqlen >= 1, "restore_dense_fwd: seqlen must be >= 1");
    const int64_t E = y_flat.size(0);
    const int64_t NC = cu_seqlens.size(0) - 1;
    TORCH_CHECK(NC >= 1, "restore_dense_fwd: cu_seqlens must have at least 2 elements");
    TORCH_CHECK(NC % dim == 0, "restore_dense_fwd: n_channels (B*D) must be divisible by dim");
    auto out_type = out_dtype_opt.value_or(input_type);
    TORCH_CHECK(out_type == at::ScalarType::Float || out_type == at::ScalarType::Half ||
                    out_type == at::ScalarType::BFloat16,
                "restore_dense_fwd: out_dtype must be fp32, fp16, or bf16");
    if (input_type == at::ScalarType::Half)
        TORCH_CHECK(out_type == at::ScalarType::Half, "restore_dense_fwd: fp16 input only supports fp16 output");
    if (input_type == at::ScalarType::BFloat16)
        TORCH_CHECK(out_type == at::ScalarType::BFloat16, "restore_dense_fwd: bf16 input only supports bf16 output");
    c10::cuda::CUDAGuard guard(y_flat.device());
    const int64_t B = NC / dim;
    auto out = torch::empty({B, seqlen, dim}, y_flat.options().dtype(out_type));
    if (bitmap != nullptr) {
        const int64_t words = (int64_t)bcm_restore_bitmap_bytes(NC, dim, seqlen) / 4;
        TORCH_CHECK(words > 0, "restore_dense_fwd_bitmap: bad sizes");
        *bitmap = torch::empty({words}, y_flat.options().dtype(at::ScalarType::Int));
        if (base_mask != nullptr) {
            const Tensor& m = *base_mask;
            TORCH_CHECK(expand >= 1 && dim % expand == 0, "restore_dense_fwd_bitmap: dim must be a multiple of expand");
            TORCH_CHECK(m.is_cuda() && m.is_contiguous() && m.device() == y_flat.device() &&
                            m.nbytes() >= (size_t)(NC / expand) * (size_t)((seqlen + 31) / 32) * 4,
                        "restore_dense_fwd_bitmap: base_mask must be the mask buffer extract_expanded_events "
                        "returned (keep_mask=True) for this stream");
            check_status(bcm_restore_dense_fwd_mask(y_flat.data_ptr(), to_bcm(input_type, "restore_dense_fwd"),
                                                    time_steps.data_ptr<int32_t>(), cu_seqlens.data_ptr<int32_t>(),
                                                    E, NC, dim, seqlen, out.data_ptr(),
                                                    to_bcm(out_type, "restore_dense_fwd"),
                                                    reinterpret_cast<const uint32_t*>(m.data_ptr()), expand,
                                                    reinterpret_cast<uint32_t*>(bitmap->data_ptr<int32_t>()),
                                                    cur_stream()),
                         "restore_dense_fwd_mask");
            return out;
        }
        check_status(bcm_restore_dense_fwd_bitmap(y_flat.data_ptr(), to_bcm(input_type, "restore_dense_fwd"),
                                                  time_steps.data_ptr<int32_t>(), cu_seqlens.data_ptr<int32_t>(),
                                                  E, NC, dim, seqlen, out.data_ptr(),
                                                  to_bcm(out_type, "restore_dense_fwd"),
                                                  reinterpret_cast<uint32_t*>(bitmap->data_ptr<int32_t>()),
                                                  cur_stream()),
                     "restore_dense_fwd_bitmap");
        return out;
    }
    check_status(bcm_restore_dense_fwd(y_flat.data_ptr(), to_bcm(input_type, "restore_dense_fwd"),
                                       time_steps.data_ptr<int32_t>(), cu_seqlens.data_ptr<int32_t>(),
                                       E, NC, dim, seqlen, out.data_ptr(),
                                       to_bcm(out_type, "restore_dense_fwd"), cur_stream()),
                 "restore_dense_fwd");
    return out;
}

Tensor restore_dense_fwd(const Tensor& y_flat, const Tensor& time_steps, const Tensor& cu_seqlens,
                         int64_t dim, int64_t seqlen, const optional<at::ScalarType> out_dtype_opt) {
    return restore_fwd_impl(y_flat, time_steps, cu_seqlens, dim, seqlen, out_dtype_opt, nullptr);
}

std::vector<Tensor> restore_dense_fwd_bitmap(const Tensor& y_flat, const Tensor& time_steps,
                                             const Tensor& cu_seqlens, int64_t dim, int64_t seqlen,
                                             const optional<at::ScalarType> out_dtype_opt,
                                             const optional<Tensor>& base_mask, int64_t expand) {
    Tensor bitmap;
    const Tensor* m = (base_mask.has_value() && base_mask->defined()) ? &*base_mask : nullptr;
    Tensor out = restore_fwd_impl(y_flat, time_steps, cu_seqlens, dim, seqlen, out_dtype_opt, &bitmap, m, expand);
    return {out, bitmap};
}

Tensor restore_dense_bwd(const Tensor& dout, const Tensor& time_steps, const Tensor& cu_seqlens,
                         int64_t dim, int64_t seqlen, bool bitmap) {
    auto input_type = dout.scalar_type();
    TORCH_CHECK(input_type == at::ScalarType::Float || input_type == at::ScalarType::Half ||
                    input_type == at::ScalarType::BFloat16,
                "restore_dense_bwd: dout must be fp32/fp16/bf16");
    TORCH_CHECK(time_steps.scalar_type() == at::ScalarType::Int, "restore_dense_bwd: time_steps must be int32");
    TORCH_CHECK(cu_seqlens.scalar_type() == at::ScalarType::Int, "restore_dense_bwd: cu_seqlens must be int32");
    TORCH_CHECK(dout.is_cuda() && time_steps.is_cuda() && cu_seqlens.is_cuda(),
                "restore_dense_bwd: all tensors must be on CUDA");
    TORCH_CHECK(dout.is_contiguous() && time_steps.is_contiguous() && cu_seqlens.is_contiguous(),
                "restore_dense_bwd: all tensors must be contiguous");
    TORCH_CHECK(dim >= 1, "restore_dense_bwd: dim must be >= 1");
    TORCH_CHECK(seqlen >= 1, "restore_dense_bwd: seqlen must be >= 1");
    const int64_t NC = cu_seqlens.size(0) - 1;
    const int64_t E = time_steps.size(0);
    TORCH_CHECK(dout.dim() == 3, "restore_dense_bwd: dout must be 3-D (B, L, D)");
    TORCH_CHECK(dout.size(1) == seqlen, "restore_dense_bwd: dout.size(1) must equal seqlen");
    TORCH_CHECK(dout.size(2) == dim, "restore_dense_bwd: dout.size(2) must equal dim (D)");
    TORCH_CHECK(dout.size(0) * dim == NC, "restore_dense_bwd: dout.size(0)*dim must equal n_channels");
    c10::cuda::CUDAGuard guard(dout.device());
    auto dy = torch::empty({E}, dout.options().dtype(at::ScalarType::Float));
    if (E == 0) return dy;
    Tensor ws = workspace(bitmap ? (int64_t)bcm_restore_workspace_bytes(NC, seqlen) : 0, dout.device());
    check_status(bcm_restore_dense_bwd(dout.data_ptr(), to_bcm(input_type, "restore_dense_bwd"),
                                       time_steps.data_ptr<int32_t>(), cu_seqlens.data_ptr<int32_t>(),
                                       E, NC, dim, seqlen, dy.data_ptr<float>(),
                                       bitmap ? ws.data_ptr() : nullptr, bitmap ? (size_t)ws.numel() : 0,
                                       cur_stream()),
                 "restore_dense_bwd");
    return dy;
}

Tensor restore_dense_bwd_bitmap(const Tensor& dout, const Tensor& time_steps, const Tensor& cu_seqlens,
                                const Tensor& bitmap, int64_t dim, int64_t seqlen) {
    auto input_type = dout.scalar_type();
    TORCH_CHECK(input_type == at::ScalarType::Float || input_type == at::ScalarType::Half ||
                    input_type == at::ScalarType::BFloat16,
                "restore_dense_bwd_bitmap: dout must be fp32/fp16/bf16");
    TORCH_CHECK(time_steps.scalar_type() == at::ScalarType::Int && cu_seqlens.scalar_type() == at::ScalarType::Int &&
                    bitmap.scalar_type() == at::ScalarType::Int,
                "restore_dense_bwd_bitmap: time_steps, cu_seqlens and bitmap must be int32");
    TORCH_CHECK(dout.is_cuda() && time_steps.is_cuda() && cu_seqlens.is_cuda() && bitmap.is_cuda(),
                "restore_dense_bwd_bitmap: all tensors must be on CUDA");
    TORCH_CHECK(dout.is_contiguous() && cu_seqlens.is_contiguous() && bitmap.is_contiguous(),
                "restore_dense_bwd_bitmap: all tensors must be contiguous");
    TORCH_CHECK(dim >= 1 && seqlen >= 1, "restore_dense_bwd_bitmap: dim and seqlen must be >= 1");
    const int64_t NC = cu_seqlens.size(0) - 1;
    const int64_t E = time_steps.size(0);
    TORCH_CHECK(dout.dim() == 3 && dout.size(1) == seqlen && dout.size(2) == dim && dout.size(0) * dim == NC,
                "restore_dense_bwd_bitmap: dout must be (B, seqlen, dim) with B*dim = n_channels");
    TORCH_CHECK(bitmap.dim() == 1 && bitmap.numel() * 4 == (int64_t)bcm_restore_bitmap_bytes(NC, dim, seqlen),
                "restore_dense_bwd_bitmap: bitmap must be the buffer restore_dense_fwd_bitmap returned for these "
                "sizes on this device");
    c10::cuda::CUDAGuard guard(dout.device());
    auto dy = torch::empty({E}, dout.options().dtype(at::ScalarType::Float));
    if (E == 0) return dy;
    check_status(bcm_restore_dense_bwd_bitmap(dout.data_ptr(), to_bcm(input_type, "restore_dense_bwd_bitmap"),
                                              time_steps.data_ptr<int32_t>(), cu_seqlens.data_ptr<int32_t>(),
                                              E, NC, dim, seqlen,
                                              reinterpret_cast<const uint32_t*>(bitmap.data_ptr<int32_t>()),
                                              dy.data_ptr<float>(), cur_stream()),
                 "restore_dense_bwd_bitmap");
    return dy;
}

// ------------------------------------------------------- block parameters ----
// (the messages name the expected shape symbolically, see check_status)
static void check_param(const Tensor& t, const char* name, int64_t n0, int64_t n1, const char* shape) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous(), "event_params: ", name,
                " must be a contiguous float32 CUDA tensor");
    if (n1 < 0) {
        TORCH_CHECK(t.dim() == 1 && t.size(0) == n0, "event_params: ", name, " must have shape ", shape);
    } else {
        TORCH_CHECK(t.dim() == 2 && t.size(0) == n0 && t.size(1) == n1, "event_params: ", name,
                    " must have shape ", shape);
    }
}

std::vector<Tensor> event_params_fwd(const Tensor& A_log, const Tensor& W_BC, const Tensor& a0, const Tensor& a1,
                                     double eps) {
    TORCH_CHECK(A_log.dim() == 2, "event_params: A_log must be 2-D (dim, dstate)");
    const int64_t dim = A_log.size(0), N = A_log.size(1);
    check_param(A_log, "A_log", dim, N, "(dim, dstate)");
    check_param(W_BC, "W_BC", dim, 2 * N, "(dim, 2*dstate)");
    check_param(a0, "a0", dim, -1, "(dim)");
    check_param(a1, "a1", dim, -1, "(dim)");
    c10::cuda::CUDAGuard guard(A_log.device());
    auto A = torch::empty_like(A_log), W_B = torch::empty_like(A_log), W_C = torch::empty_like(A_log);
    auto dt_idle = torch::empty_like(a0), dt_active = torch::empty_like(a1);
    check_status(bcm_event_params_fwd(A_log.data_ptr<float>(), W_BC.data_ptr<float>(), a0.data_ptr<float>(),
                                      a1.data_ptr<float>(), dim, N, (float)eps, A.data_ptr<float>(),
                                      W_B.data_ptr<float>(), W_C.data_ptr<float>(), dt_idle.data_ptr<float>(),
                                      dt_active.data_ptr<float>(), cur_stream()),
                 "event_params_fwd");
    return {A, W_B, W_C, dt_idle, dt_active};
}

// gradients given as None are zero
std::vector<Tensor> event_params_bwd(const Tensor& A, const Tensor& a0, const Tensor& a1, const optional<Tensor>& dA,
                                     const optional<Tensor>& dW_B, const optional<Tensor>& dW_C,
                                     const optional<Tensor>& ddt_idle, const optional<Tensor>& ddt_active) {
    TORCH_CHECK(A.dim() == 2, "event_params: A must be 2-D (dim, dstate)");
    const int64_t dim = A.size(0), N = A.size(1);
    check_param(A, "A", dim, N, "(dim, dstate)");
    check_param(a0, "a0", dim, -1, "(dim)");
    check_param(a1, "a1", dim, -1, "(dim)");
    auto ptr = [&](const optional<Tensor>& t, const char* name, int64_t n1, const char* shape) -> const float* {
        if (!t.has_value()) return nullptr;
        check_param(*t, name, dim, n1, shape);
        return t->data_ptr<float>();
    };
    const float* pdA = ptr(dA, "dA", N, "(dim, dstate)");
    const float* pdB = ptr(dW_B, "dW_B", N, "(dim, dstate)");
    const float* pdC = ptr(dW_C, "dW_C", N, "(dim, dstate)");
    const float* pdi = ptr(ddt_idle, "ddt_idle", -1, "(dim)");
    const float* pda = ptr(ddt_active, "ddt_active", -1, "(dim)");
    c10::cuda::CUDAGuard guard(A.device());
    auto dA_log = torch::empty_like(A);
    auto dW_BC = torch::empty({dim, 2 * N}, A.options());
    auto da0 = torch::empty_like(a0), da1 = torch::empty_like(a1);
    check_status(bcm_event_params_bwd(A.data_ptr<float>(), a0.data_ptr<float>(), a1.data_ptr<float>(), pdA, pdB, pdC,
                                      pdi, pda, dim, N, dA_log.data_ptr<float>(), dW_BC.data_ptr<float>(),
                                      da0.data_ptr<float>(), da1.data_ptr<float>(), cur_stream()),
                 "event_params_bwd");
    return {dA_log, dW_BC, da0, da1};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.attr("abi_version") = bcm_abi_version();
    // selective_scan_cuda
    m.def("fwd", &selective_scan_fwd, "dense selective scan forward");
    m.def("bwd", &selective_scan_bwd, "dense selective scan backward");
    m.def("fwd_flat_ch", &selective_scan_fwd_flat_ch, py::arg("u_flat"), py::arg("k_flat"),
          py::arg("cu_seqlens"), py::arg("max_seqlen"), py::arg("dt_idle"), py::arg("dt_active"),
          py::arg("A"), py::arg("B"), py::arg("C"), py::arg("D") = py::none(),
          py::arg("z") = py::none(), py::arg("tile_offsets") = py::none(),
          py::arg("tile_chunk_size") = 0, py::arg("is_depthwise_bc") = false,
          py::arg("pw_B") = py::none(), py::arg("pw_C") = py::none(),
          "Selective scan forward (flat per-channel, jagged layout)");
    m.def("fwd_flat_ch_ckpt", &selective_scan_fwd_flat_ch_ckpt, py::arg("u_flat"), py::arg("k_flat"),
          py::arg("cu_seqlens"), py::arg("max_seqlen"), py::arg("dt_idle"), py::arg("dt_active"),
          py::arg("A"), py::arg("B"), py::arg("C"), py::arg("D") = py::none(),
          py::arg("z") = py::none(), py::arg("tile_offsets") = py::none(),
          py::arg("tile_chunk_size") = 0, py::arg("is_depthwise_bc") = false,
          py::arg("pw_B") = py::none(), py::arg("pw_C") = py::none(),
          "fwd_flat_ch whose result ends with the state checkpoints for bwd_flat_ch(ckpt=...) "
          "(an empty tensor where they do not apply)");
    m.def("bwd_flat_ch", &selective_scan_bwd_flat_ch, py::arg("u_flat"), py::arg("k_flat"),
          py::arg("cu_seqlens"), py::arg("max_seqlen"), py::arg("dt_idle"), py::arg("dt_active"),
          py::arg("A"), py::arg("B"), py::arg("C"), py::arg("dout_flat"), py::arg("x"),
          py::arg("D") = py::none(), py::arg("z") = py::none(), py::arg("out") = py::none(),
          py::arg("tile_offsets") = py::none(), py::arg("tile_chunk_size") = 0,
          py::arg("is_depthwise_bc") = false, py::arg("pw_B") = py::none(),
          py::arg("pw_C") = py::none(), py::arg("ckpt") = py::none(),
          "Selective scan backward (flat per-channel, jagged layout); ckpt: the checkpoints "
          "fwd_flat_ch_ckpt returned for the same inputs");
    // extract_events_cuda
    m.def("extract_events", &extract_events_fwd, "bool mask -> (ch_ids, t_steps, k_flat, cu_seqlens, max_seqlen, head_flags)");
    m.def("extract_base_events", &extract_base_events_fwd,
          "float base_input + threshold -> (base_ch_ids, base_t_steps, base_k_flat, base_cu_seqlens, base_counts, base_max_seqlen)");
    m.def("extract_base_events_host_max", &extract_base_events_host_max, py::arg("x"), py::arg("threshold"),
          py::arg("bld") = false,
          "extract_base_events (bld: from the (B, L, d_model) layout) -> (6 outputs, max count as a host int)");
    m.def("extract_expanded_events", &extract_expanded_events, py::arg("x"), py::arg("threshold"),
          py::arg("expand"), py::arg("bld") = false, py::arg("x_conv") = py::none(),
          py::arg("feature_thresholds") = py::none(), py::arg("keep_mask") = false,
          "extract_base_events then expand_base_events in one fill pass -> ((ch, t, k, cu, max[, x_flat]), "
          "max count as a host int); bld: from the (B, L, d_model) layout; x_conv (B, d_model*expand, L): "
          "also gather_events_fwd of it at the stream (x_flat); feature_thresholds (d_model) float32 with bld: "
          "feature j fires above feature_thresholds[j] instead of threshold; keep_mask: the buffer holding the "
          "threshold mask is appended last (for restore_dense_fwd_bitmap(base_mask=))");
    m.def("extract_base_events_bld", &extract_base_events_bld_fwd, py::arg("x"), py::arg("threshold"),
          "extract_base_events from the (B, L, d_model) layout: same 6 outputs, no transposed copy");
    m.def("conv_events_fwd", &conv_events_fwd, py::arg("x"), py::arg("weight"), py::arg("bias"),
          py::arg("channel_ids"), py::arg("time_steps"),
          "silu(causal depthwise conv1d(x)) evaluated at the events -> [u_flat]");
    m.def("conv_events_bwd", &conv_events_bwd, py::arg("x"), py::arg("weight"), py::arg("bias"),
          py::arg("time_steps"), py::arg("cu_seqlens"), py::arg("grad"),
          "backward of conv_events_fwd -> [dx (B, D, L), dweight (D, K) fp32, dbias (D) fp32]");
    m.def("expand_base_events", &expand_base_events_fwd,
          "expand the base event stream by `expand` (repeat_interleave order)");
    m.def("gather_events_fwd", &gather_events_fwd, "gather x[B,D,L] at (channel_ids, time_steps)");
    m.def("gather_events_bwd", &gather_events_bwd, "scatter-store backward of gather_events_fwd");
    // restore_dense_cuda_nodecay
    m.def("restore_dense_fwd", &restore_dense_fwd, py::arg("y_flat"), py::arg("time_steps"),
          py::arg("cu_seqlens"), py::arg("dim"), py::arg("seqlen"), py::arg("out_dtype") = py::none(),
          "Zero-order-hold restore (B, L, D) from flat events");
    m.def("gather_events_bwd_rows", &gather_events_bwd_rows, py::arg("grad_x"), py::arg("time_steps"),
          py::arg("cu_seqlens"), py::arg("n_channels"), py::arg("seqlen"),
          "gather_events_bwd for a stream in extraction order, rows from cu_seqlens -> dx [NC, L]");
    m.def("event_decode_step", &event_decode_step, py::arg("x"), py::arg("spikes"), py::arg("threshold"),
          py::arg("dt_idle"), py::arg("dt_active"), py::arg("A"), py::arg("W_B"), py::arg("W_C"),
          py::arg("D"), py::arg("eta"), py::arg("counters"), py::arg("held"),
          py::arg("conv_state") = py::none(), py::arg("conv_weight") = py::none(), py::arg("conv_bias") = py::none(),
          "One token of the event path for every channel (state updated in place) -> y (B, D)");
    m.def("restore_dense_fwd_bitmap", &restore_dense_fwd_bitmap, py::arg("y_flat"), py::arg("time_steps"),
          py::arg("cu_seqlens"), py::arg("dim"), py::arg("seqlen"), py::arg("out_dtype") = py::none(),
          py::arg("base_mask") = py::none(), py::arg("expand") = 1,
          "restore_dense_fwd that also returns the event bitmap (the first B*ceil(L/32)*dim int32 words, "
          "layout [B, ceil(L/32), dim]) and the sweep's start indices, consumed by restore_dense_bwd_bitmap; "
          "base_mask (the mask buffer of extract_expanded_events(keep_mask=True) for this stream, dim = "
          "d_model*expand, seqlen <= 4095): the bitmap is transposed from it instead of built from the events");
    m.def("restore_dense_bwd_bitmap", &restore_dense_bwd_bitmap, py::arg("dout"), py::arg("time_steps"),
          py::arg("cu_seqlens"), py::arg("bitmap"), py::arg("dim"), py::arg("seqlen"),
          "Backward of restore_dense_fwd from the forward's event bitmap; returns dy_flat (float32)");
    m.def("restore_dense_bwd", &restore_dense_bwd, py::arg("dout"), py::arg("time_steps"),
          py::arg("cu_seqlens"), py::arg("dim"), py::arg("seqlen"), py::arg("bitmap") = true,
          "Backward of restore_dense_fwd; returns dy_flat (float32).  bitmap=False runs the "
          "windowed kernel (no workspace) instead of the event-bitmap one (same result up to fp32 rounding)");
    // block parameter transforms (no reference binding: PyTorch ops in Mamba.forward)
    m.def("event_params_fwd", &event_params_fwd, py::arg("A_log"), py::arg("W_BC"), py::arg("a0"), py::arg("a1"),
          py::arg("eps"),
          "-> [A = -exp(A_log), W_B, W_C (the halves of W_BC), softplus(a0) + eps, softplus(a1) + eps]");
    m.def("event_params_bwd", &event_params_bwd, py::arg("A"), py::arg("a0"), py::arg("a1"), py::arg("dA"),
          py::arg("dW_B"), py::arg("dW_C"), py::arg("ddt_idle"), py::arg("ddt_active"),
          "backward of event_params_fwd (None gradients are zero) -> [dA_log, dW_BC, da0, da1]");
}
