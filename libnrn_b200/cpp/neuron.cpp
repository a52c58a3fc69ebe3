// neuron.cpp -- LIF, AdEx and Izhikevich models of the nrn:: API.
//
// Same structs, lifecycle and operations tables as the reference
// (src/neuron/lif.cpp, adex.cpp, izhikevich.cpp).  The model's tensors are
// created on the current CUDA device (CPU only where no GPU exists, for
// construction and inspection); *_forward runs nrn_cuda_pop_step, which
// updates the state tensors in place on the current CUDA stream.
#include <nrn/neuron/adex.h>
#include <nrn/neuron/izhikevich.h>
#include <nrn/neuron/lif.h>

#include "support.h"

namespace nrn {
namespace neuron {

using detail::cuda_f32;

namespace {

torch::TensorOptions model_options(torch::Dtype dtype, const char* who) {
    TORCH_CHECK(dtype == torch::kFloat32, who, ": libnrn_b200 models are float32");
    return torch::TensorOptions().dtype(dtype).device(detail::default_device());
}

void set_params(nrn_pop_step_t& a, std::initializer_list<torch::Tensor*> ps, int64_t n, const char* where) {
    int k = 0;
    for (torch::Tensor* p : ps) {
        a.param[k] = cuda_f32(*p, n, "parameter", where);
        ++k;
    }
}

void run(nrn_pop_step_t& a, const torch::Tensor& like, const char* where) {
    detail::check(nrn_cuda_pop_step(&a, detail::stream_of(like)), where);
}

const char* kLifVars[] = {"v", "spike", "refractory", "I_syn"};
const char* kAdexVars[] = {"v", "w", "spike", "refractory", "I_syn"};
const char* kIzhVars[] = {"v", "u", "spike", "I_syn"};

}  // namespace

// ---------------------------------------------------------------- LIF ----

nrn_ops lif_ops = {lif_forward, lif_reset, lif_state_vars, lif_size, lif_to_device};

LIFNeuron* lif_create(int64_t n, LIFOptions opts) {
    TORCH_CHECK(n >= 0, "lif_create: n must be >= 0");
    auto* m = new LIFNeuron();
    m->n = n;
    m->options = opts;
    auto o = model_options(opts.dtype(), "lif_create");
    m->v = torch::full({n}, opts.v_rest(), o);
    m->spike = torch::zeros({n}, o);
    m->refractory = torch::zeros({n}, o);
    m->I_syn = torch::zeros({n}, o);
    m->v_rest = torch::full({n}, opts.v_rest(), o);
    m->v_thresh = torch::full({n}, opts.v_thresh(), o);
    m->v_reset = torch::full({n}, opts.v_reset(), o);
    m->tau_m = torch::full({n}, opts.tau_m(), o);
    m->tau_ref = torch::full({n}, opts.tau_ref(), o);
    m->c_m = torch::full({n}, opts.c_m(), o);
    m->i_bg = torch::full({n}, opts.i_bg(), o);
    return m;
}

void lif_destroy(LIFNeuron* m) { delete m; }

void lif_forward(void* self, State& state, double /*t*/, double dt) {
    auto* m = static_cast<LIFNeuron*>(self);
    const char* w = "lif_forward";
    if (m->n > 0) {
        nrn_pop_step_t a{};
        a.model = NRN_MODEL_LIF;
        a.n = static_cast<int32_t>(m->n);
        a.dt = dt;
        a.v = cuda_f32(m->v, m->n, "v", w);
        a.refractory = cuda_f32(m->refractory, m->n, "refractory", w);
        a.spike = cuda_f32(m->spike, m->n, "spike", w);
        a.i_syn = cuda_f32(m->I_syn, m->n, "I_syn", w);
        set_params(a, {&m->v_rest, &m->v_thresh, &m->v_reset, &m->tau_m, &m->tau_ref, &m->c_m, &m->i_bg}, m->n, w);
        run(a, m->v, w);
    }
    state_set(state, "v", m->v);
    state_set(state, "spike", m->spike);
    state_set(state, "refractory", m->refractory);
    state_set(state, "I_syn", m->I_syn);
}

void lif_reset(void* self) {
    auto* m = static_cast<LIFNeuron*>(self);
    m->v.fill_(m->options.v_rest());
    m->spike.zero_();
    m->refractory.zero_();
    m->I_syn.zero_();
}

const char** lif_state_vars(void*, int* count) {
    *count = 4;
    return kLifVars;
}

int64_t lif_size(void* self) { return static_cast<LIFNeuron*>(self)->n; }

void lif_to_device(void* self, torch::Device device) {
    auto* m = static_cast<LIFNeuron*>(self);
    for (torch::Tensor* t : {&m->v, &m->spike, &m->refractory, &m->I_syn, &m->v_rest, &m->v_thresh, &m->v_reset,
                             &m->tau_m, &m->tau_ref, &m->c_m, &m->i_bg})
        *t = t->to(device);
}

// --------------------------------------------------------------- AdEx ----

nrn_ops adex_ops = {adex_forward, adex_reset, adex_state_vars, adex_size, adex_to_device};

AdExNeuron* adex_create(int64_t n, AdExOptions opts) {
    TORCH_CHECK(n >= 0, "adex_create: n must be >= 0");
    auto* m = new AdExNeuron();
    m->n = n;
    m->options = opts;
    auto o = model_options(opts.dtype(), "adex_create");
    m->v = torch::full({n}, opts.v_rest(), o);
    m->w = torch::zeros({n}, o);
    m->spike = torch::zeros({n}, o);
    m->refractory = torch::zeros({n}, o);
    m->I_syn = torch::zeros({n}, o);
    m->v_rest = torch::full({n}, opts.v_rest(), o);
    m->v_thresh = torch::full({n}, opts.v_thresh(), o);
    m->v_reset = torch::full({n}, opts.v_reset(), o);
    m->v_peak = torch::full({n}, opts.v_peak(), o);
    m->tau_m = torch::full({n}, opts.tau_m(), o);
    m->tau_w = torch::full({n}, opts.tau_w(), o);
    m->tau_ref = torch::full({n}, opts.tau_ref(), o);
    m->c_m = torch::full({n}, opts.c_m(), o);
    m->g_l = torch::full({n}, opts.g_l(), o);
    m->a = torch::full({n}, opts.a(), o);
    m->b = torch::full({n}, opts.b(), o);
    m->delta_t = torch::full({n}, opts.delta_t(), o);
    m->i_bg = torch::full({n}, opts.i_bg(), o);
    return m;
}

void adex_destroy(AdExNeuron* m) { delete m; }

void adex_forward(void* self, State& state, double /*t*/, double dt) {
    auto* m = static_cast<AdExNeuron*>(self);
    const char* w = "adex_forward";
    if (m->n > 0) {
        nrn_pop_step_t a{};
        a.model = NRN_MODEL_ADEX;
        a.n = static_cast<int32_t>(m->n);
        a.dt = dt;
        a.v = cuda_f32(m->v, m->n, "v", w);
        a.aux = cuda_f32(m->w, m->n, "w", w);
        a.refractory = cuda_f32(m->refractory, m->n, "refractory", w);
        a.spike = cuda_f32(m->spike, m->n, "spike", w);
        a.i_syn = cuda_f32(m->I_syn, m->n, "I_syn", w);
        set_params(a, {&m->v_rest, &m->v_thresh, &m->v_reset, &m->v_peak, &m->tau_m, &m->tau_w, &m->tau_ref,
                       &m->c_m, &m->g_l, &m->a, &m->b, &m->delta_t, &m->i_bg},
                   m->n, w);
        run(a, m->v, w);
    }
    state_set(state, "v", m->v);
    state_set(state, "w", m->w);
    state_set(state, "spike", m->spike);
    state_set(state, "refractory", m->refractory);
    state_set(state, "I_syn", m->I_syn);
}

void adex_reset(void* self) {
    auto* m = static_cast<AdExNeuron*>(self);
    m->v.fill_(m->options.v_rest());
    m->w.zero_();
    m->spike.zero_();
    m->refractory.zero_();
    m->I_syn.zero_();
}

const char** adex_state_vars(void*, int* count) {
    *count = 5;
    return kAdexVars;
}

int64_t adex_size(void* self) { return static_cast<AdExNeuron*>(self)->n; }

void adex_to_device(void* self, torch::Device device) {
    auto* m = static_cast<AdExNeuron*>(self);
    for (torch::Tensor* t : {&m->v, &m->w, &m->spike, &m->refractory, &m->I_syn, &m->v_rest, &m->v_thresh,
                             &m->v_reset, &m->v_peak, &m->tau_m, &m->tau_w, &m->tau_ref, &m->c_m, &m->g_l, &m->a,
                             &m->b, &m->delta_t, &m->i_bg})
        *t = t->to(device);
}

// --------------------------------------------------------- Izhikevich ----

nrn_ops izh_ops = {izh_forward, izh_reset, izh_state_vars, izh_size, izh_to_device};

IzhikevichNeuron* izh_create(int64_t n, IzhikevichOptions opts) {
    TORCH_CHECK(n >= 0, "izh_create: n must be >= 0");
    auto* m = new IzhikevichNeuron();
    m->n = n;
    m->options = opts;
    auto o = model_options(opts.dtype(), "izh_create");
    m->v = torch::full({n}, opts.v_init(), o);
    // u starts at b * v_init (the reference ignores u_init, src/neuron/izhikevich.cpp:46)
    m->u = torch::full({n}, opts.b() * opts.v_init(), o);
    m->spike = torch::zeros({n}, o);
    m->I_syn = torch::zeros({n}, o);
    m->a = torch::full({n}, opts.a(), o);
    m->b = torch::full({n}, opts.b(), o);
    m->c = torch::full({n}, opts.c(), o);
    m->d = torch::full({n}, opts.d(), o);
    m->v_peak = torch::full({n}, opts.v_peak(), o);
    return m;
}

void izh_destroy(IzhikevichNeuron* m) { delete m; }

void izh_forward(void* self, State& state, double /*t*/, double dt) {
    auto* m = static_cast<IzhikevichNeuron*>(self);
    const char* w = "izh_forward";
    if (m->n > 0) {
        nrn_pop_step_t a{};
        a.model = NRN_MODEL_IZH;
        a.n = static_cast<int32_t>(m->n);
        a.dt = dt;
        a.v = cuda_f32(m->v, m->n, "v", w);
        a.aux = cuda_f32(m->u, m->n, "u", w);
        a.spike = cuda_f32(m->spike, m->n, "spike", w);
        a.i_syn = cuda_f32(m->I_syn, m->n, "I_syn", w);
        set_params(a, {&m->a, &m->b, &m->c, &m->d, &m->v_peak}, m->n, w);
        run(a, m->v, w);
    }
    state_set(state, "v", m->v);
    state_set(state, "u", m->u);
    state_set(state, "spike", m->spike);
    state_set(state, "I_syn", m->I_syn);
}

void izh_reset(void* self) {
    auto* m = static_cast<IzhikevichNeuron*>(self);
    m->v.fill_(m->options.v_init());
    m->u.fill_(m->options.b() * m->options.v_init());
    m->spike.zero_();
    m->I_syn.zero_();
}

const char** izh_state_vars(void*, int* count) {
    *count = 4;
    return kIzhVars;
}

int64_t izh_size(void* self) { return static_cast<IzhikevichNeuron*>(self)->n; }

void izh_to_device(void* self, torch::Device device) {
    auto* m = static_cast<IzhikevichNeuron*>(self);
    for (torch::Tensor* t : {&m->v, &m->u, &m->spike, &m->I_syn, &m->a, &m->b, &m->c, &m->d, &m->v_peak})
        *t = t->to(device);
}

}  // namespace neuron
}  // namespace nrn
