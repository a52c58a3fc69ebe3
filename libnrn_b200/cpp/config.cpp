// config.cpp -- YAML configuration of a Region or a Simulation.
//
// The reference declares nrn::config::load / load_region
// (include/nrn/config/config.h) and throws from both
// (src/config/config.cpp:8-18); its design notes sketch the file layout
// (simulation / populations / connections).  This loader reads that layout
// with the library's own small YAML reader (block mappings and sequences,
// flow sequences and mappings, comments, quoted strings -- the subset these
// files use; anchors, multi-line scalars and tags are refused) and builds
// the objects through the public nrn:: API:
//
//   name: cortex                    # Region name (default "region")
//   seed: 42                        # torch::manual_seed before connectivity
//   simulation:                     # load() only; SimulationOptions fields
//     dt_fast: 0.1ms
//     dt_slow: 1ms
//     duration: 1s
//     device: cuda                  # or cpu
//   populations:
//     - name: exc
//       model: LIF                  # LIF | AdEx | Izhikevich
//       count: 8000
//       params: {tau_m: 20ms, v_thresh: 20mV}   # the model's option fields
//   connections:
//     - source: exc
//       target: exc
//       topology: random            # random | distance_dependent
//       probability: 0.1            # or sigma / max_distance / min_probability
//       weight: 250pA               # ConnectOptions weight_scale
//       block_size: 64
//       synapse: static             # static | exponential | double_exponential | AMPA
//       synapse_params: {tau_decay: 5ms}
//       plasticity: stdp            # optional
//       plasticity_params: {a_plus: 0.01, w_max: 500pA}
//   record:                         # load() only: sim_record
//     - population: exc
//       variables: [spike]
//
// Quantities take SI unit suffixes (s ms us, V mV, A nA pA, F nF pF, S uS nS,
// m mm um, Hz); bare numbers are SI.  Errors (syntax, unknown keys, unknown
// populations or models) throw std::runtime_error with the file and line,
// the reference's error type for this API.
#include <nrn/config/config.h>
#include <nrn/connectivity/connect.h>
#include <nrn/connectivity/topology/distance_dependent.h>
#include <nrn/connectivity/topology/random.h>
#include <nrn/neuron/adex.h>
#include <nrn/neuron/izhikevich.h>
#include <nrn/neuron/lif.h>
#include <nrn/plasticity/stdp.h>
#include <nrn/synapse/synapse.h>

#include <cctype>
#include <cmath>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace nrn {
namespace config {

namespace {

// ----------------------------------------------------------------- YAML ----

struct Node {
    enum Kind { Null, Scalar, Map, Seq } kind = Null;
    std::string text;                                   // Scalar
    std::vector<std::pair<std::string, Node>> map;      // Map, in file order
    std::vector<Node> seq;                              // Seq
    int line = 0;
    const Node* get(const std::string& k) const {
        for (const auto& kv : map)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct Line {
    int indent;
    std::string text;   // without indentation and comment
    int no;
};

[[noreturn]] void fail_at(const std::string& file, int line, const std::string& what) {
    throw std::runtime_error("nrn::config: " + file + ":" + std::to_string(line) + ": " + what);
}

std::string trim(const std::string& s) {
    size_t a = 0, b = s.size();
    while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
    while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
    return s.substr(a, b - a);
}

// The text before an unquoted '#'.
std::string strip_comment(const std::string& s) {
    char q = 0;
    for (size_t i = 0; i < s.size(); ++i) {
        const char c = s[i];
        if (q) {
            if (c == q) q = 0;
        } else if (c == '"' || c == '\'') {
            q = c;
        } else if (c == '#' && (i == 0 || std::isspace(static_cast<unsigned char>(s[i - 1])))) {
            return s.substr(0, i);
        }
    }
    return s;
}

class Reader {
  public:
    Reader(const std::string& file, const std::string& text) : file_(file) {
        std::istringstream in(text);
        std::string raw;
        int no = 0;
        while (std::getline(in, raw)) {
            ++no;
            if (!raw.empty() && raw.back() == '\r') raw.pop_back();
            if (raw.find('\t') != std::string::npos && trim(strip_comment(raw)).size())
                fail_at(file_, no, "tab characters are not allowed in indentation");
            const std::string body = strip_comment(raw);
            const std::string t = trim(body);
            if (t.empty() || t == "---") continue;
            if (t == "...") break;
            int ind = 0;
            while (ind < static_cast<int>(body.size()) && body[ind] == ' ') ++ind;
            lines_.push_back({ind, t, no});
        }
    }

    Node parse() {
        size_t i = 0;
        if (lines_.empty()) return Node{};
        Node n = block(i, lines_[0].indent);
        if (i != lines_.size()) fail_at(file_, lines_[i].no, "unexpected indentation");
        return n;
    }

  private:
    // A block starting at line i whose lines are indented by `ind`.
    Node block(size_t& i, int ind) {
        const bool seq = lines_[i].text.rfind("- ", 0) == 0 || lines_[i].text == "-";
        Node n;
        n.kind = seq ? Node::Seq : Node::Map;
        n.line = lines_[i].no;
        while (i < lines_.size() && lines_[i].indent == ind) {
            const Line& L = lines_[i];
            const bool is_item = L.text.rfind("- ", 0) == 0 || L.text == "-";
            if (is_item != seq) {
                if (seq) break;   // a sequence at its key's indentation ends at the next key
                fail_at(file_, L.no, "mixed sequence and mapping entries");
            }
            if (seq) {
                std::string rest = L.text == "-" ? "" : trim(L.text.substr(2));
                if (rest.empty()) {
                    ++i;
                    if (i < lines_.size() && lines_[i].indent > ind) n.seq.push_back(block(i, lines_[i].indent));
                    else n.seq.push_back(Node{});
                } else if (split_key(rest).first.size()) {
                    // "- key: value" starts a mapping whose further keys are
                    // indented to the column after "- "
                    Line first = L;
                    first.indent = ind + 2;
                    first.text = rest;
                    lines_[i] = first;
                    n.seq.push_back(block(i, ind + 2));
                } else {
                    n.seq.push_back(value(rest, L.no));
                    ++i;
                }
            } else {
                auto kv = split_key(L.text);
                if (kv.first.empty()) fail_at(file_, L.no, "expected 'key: value'");
                for (const auto& e : n.map)
                    if (e.first == kv.first) fail_at(file_, L.no, "duplicate key '" + kv.first + "'");
                ++i;
                if (kv.second.empty()) {
                    const bool same_seq = i < lines_.size() && lines_[i].indent == ind &&
                                          (lines_[i].text.rfind("- ", 0) == 0 || lines_[i].text == "-");
                    if (i < lines_.size() && (lines_[i].indent > ind || same_seq))
                        n.map.emplace_back(kv.first, block(i, lines_[i].indent));
                    else n.map.emplace_back(kv.first, Node{});
                } else {
                    n.map.emplace_back(kv.first, value(kv.second, L.no));
                }
            }
        }
        if (i < lines_.size() && lines_[i].indent > ind) fail_at(file_, lines_[i].no, "unexpected indentation");
        return n;
    }

    // ("key", "value") of "key: value" (key may be quoted), or ("", "").
    std::pair<std::string, std::string> split_key(const std::string& t) const {
        char q = 0;
        for (size_t i = 0; i < t.size(); ++i) {
            const char c = t[i];
            if (q) {
                if (c == q) q = 0;
            } else if ((c == '"' || c == '\'') && i == 0) {
                q = c;
            } else if (c == '[' || c == '{') {
                return {"", ""};
            } else if (c == ':' && (i + 1 == t.size() || t[i + 1] == ' ')) {
                return {unquote(trim(t.substr(0, i))), trim(t.substr(i + 1))};
            }
        }
        return {"", ""};
    }

    std::string unquote(const std::string& s) const {
        if (s.size() >= 2 && (s.front() == '"' || s.front() == '\'') && s.back() == s.front())
            return s.substr(1, s.size() - 2);
        return s;
    }

    Node value(const std::string& s, int no) {
        if (s == "|" || s == ">" || s[0] == '&' || s[0] == '*' || s[0] == '!')
            fail_at(file_, no, "unsupported YAML feature: '" + s + "'");
        size_t p = 0;
        Node n = flow(s, p, no);
        while (p < s.size() && s[p] == ' ') ++p;
        if (p != s.size()) fail_at(file_, no, "trailing characters after a value");
        return n;
    }

    Node flow(const std::string& s, size_t& p, int no) {
        while (p < s.size() && s[p] == ' ') ++p;
        Node n;
        n.line = no;
        if (p < s.size() && (s[p] == '[' || s[p] == '{')) {
            const char close = s[p] == '[' ? ']' : '}';
            const bool is_map = s[p] == '{';
            n.kind = is_map ? Node::Map : Node::Seq;
            ++p;
            while (true) {
                while (p < s.size() && s[p] == ' ') ++p;
                if (p < s.size() && s[p] == close) {
                    ++p;
                    break;
                }
                if (is_map) {
                    size_t c = p;
                    while (c < s.size() && s[c] != ':') ++c;
                    if (c >= s.size()) fail_at(file_, no, "expected 'key: value' in a flow mapping");
                    const std::string k = unquote(trim(s.substr(p, c - p)));
                    p = c + 1;
                    n.map.emplace_back(k, flow(s, p, no));
                } else {
                    n.seq.push_back(flow(s, p, no));
                }
                while (p < s.size() && s[p] == ' ') ++p;
                if (p < s.size() && s[p] == ',') {
                    ++p;
                    continue;
                }
                if (p < s.size() && s[p] == close) {
                    ++p;
                    break;
                }
                fail_at(file_, no, std::string("expected ',' or '") + close + "'");
            }
            return n;
        }
        size_t b = p;
        if (p < s.size() && (s[p] == '"' || s[p] == '\'')) {
            const char q = s[p++];
            while (p < s.size() && s[p] != q) ++p;
            if (p >= s.size()) fail_at(file_, no, "unterminated string");
            n.kind = Node::Scalar;
            n.text = s.substr(b + 1, p - b - 1);
            ++p;
            return n;
        }
        while (p < s.size() && s[p] != ',' && s[p] != ']' && s[p] != '}') ++p;
        n.kind = Node::Scalar;
        n.text = trim(s.substr(b, p - b));
        if (n.text == "~" || n.text == "null") n.kind = Node::Null;
        return n;
    }

    std::string file_;
    std::vector<Line> lines_;
};

// --------------------------------------------------------------- values ----

struct Ctx {
    std::string file;
};

double quantity(const Ctx& c, const Node& n, const std::string& what) {
    if (n.kind != Node::Scalar) fail_at(c.file, n.line, what + ": expected a number");
    const std::string& s = n.text;
    size_t used = 0;
    double v = 0.0;
    try {
        v = std::stod(s, &used);
    } catch (...) {
        fail_at(c.file, n.line, what + ": '" + s + "' is not a number");
    }
    const std::string unit = trim(s.substr(used));
    static const std::map<std::string, double> scale = {
        {"", 1.0},     {"s", 1.0},     {"ms", 1e-3},  {"us", 1e-6}, {"V", 1.0},   {"mV", 1e-3},
        {"A", 1.0},    {"nA", 1e-9},   {"pA", 1e-12}, {"F", 1.0},   {"nF", 1e-9}, {"pF", 1e-12},
        {"S", 1.0},    {"uS", 1e-6},   {"nS", 1e-9},  {"m", 1.0},   {"mm", 1e-3}, {"um", 1e-6},
        {"Hz", 1.0}};
    auto it = scale.find(unit);
    if (it == scale.end()) fail_at(c.file, n.line, what + ": unknown unit '" + unit + "'");
    if (!std::isfinite(v)) fail_at(c.file, n.line, what + ": not finite");
    return v * it->second;
}

int64_t integer(const Ctx& c, const Node& n, const std::string& what) {
    const double v = quantity(c, n, what);
    if (v != std::floor(v)) fail_at(c.file, n.line, what + ": expected an integer");
    return static_cast<int64_t>(v);
}

bool boolean(const Ctx& c, const Node& n, const std::string& what) {
    if (n.kind == Node::Scalar && (n.text == "true" || n.text == "True" || n.text == "yes")) return true;
    if (n.kind == Node::Scalar && (n.text == "false" || n.text == "False" || n.text == "no")) return false;
    fail_at(c.file, n.line, what + ": expected true or false");
}

std::string text(const Ctx& c, const Node& n, const std::string& what) {
    if (n.kind != Node::Scalar) fail_at(c.file, n.line, what + ": expected a string");
    return n.text;
}

const Node& need(const Ctx& c, const Node& m, const std::string& key) {
    const Node* n = m.get(key);
    if (n == nullptr) fail_at(c.file, m.line, "missing key '" + key + "'");
    return *n;
}

// Applies a mapping of option fields; unknown keys are errors.
using Setter = std::function<void(const Node&)>;
void apply(const Ctx& c, const Node* m, const std::map<std::string, Setter>& fields, const std::string& what) {
    if (m == nullptr || m->kind == Node::Null) return;
    if (m->kind != Node::Map) fail_at(c.file, m->line, what + ": expected a mapping");
    for (const auto& kv : m->map) {
        auto it = fields.find(kv.first);
        if (it == fields.end()) fail_at(c.file, kv.second.line, what + ": unknown field '" + kv.first + "'");
        it->second(kv.second);
    }
}

void check_keys(const Ctx& c, const Node& m, std::initializer_list<const char*> allowed, const std::string& what) {
    for (const auto& kv : m.map) {
        bool ok = false;
        for (const char* a : allowed) ok = ok || kv.first == a;
        if (!ok) fail_at(c.file, kv.second.line, what + ": unknown key '" + kv.first + "'");
    }
}

#define NRN_Q(Opt, field) {#field, [&](const Node& n) { o.field(quantity(c, n, what + "." #field)); }}

// ---------------------------------------------------------------- build ----

// A population and the neuron model it does not own, released together.
template <class M>
struct PopHolder {
    std::shared_ptr<Population> pop;
    M* model = nullptr;
    void (*destroy)(M*) = nullptr;
    ~PopHolder() {
        pop.reset();
        if (model && destroy) destroy(model);
    }
};

template <class M>
std::shared_ptr<Population> own_population(const std::string& name, M* model, NrnModule mod, int64_t n,
                                           void (*destroy)(M*), torch::Device dev) {
    auto h = std::make_shared<PopHolder<M>>();
    h->model = model;
    h->destroy = destroy;
    h->pop = std::shared_ptr<Population>(population_create(name, mod, n, dev), population_destroy);
    return std::shared_ptr<Population>(h, h->pop.get());
}

// A connection with its synapse module and plasticity state, released together.
struct ConnHolder {
    std::shared_ptr<Connection> conn;
    std::function<void()> release;
    ~ConnHolder() {
        conn.reset();
        if (release) release();
    }
};

torch::Device device_of(const Ctx& c, const Node* sim) {
    if (sim && sim->get("device")) {
        const std::string d = text(c, *sim->get("device"), "simulation.device");
        if (d == "cpu") return torch::kCPU;
        if (d != "cuda") fail_at(c.file, sim->get("device")->line, "simulation.device: cpu or cuda");
    }
    return torch::kCUDA;
}

std::shared_ptr<Population> make_population(const Ctx& c, const Node& p, torch::Device dev) {
    check_keys(c, p, {"name", "model", "count", "params"}, "population");
    const std::string name = text(c, need(c, p, "name"), "population.name");
    const std::string model = text(c, need(c, p, "model"), "population.model");
    const int64_t n = integer(c, need(c, p, "count"), "population.count");
    if (n <= 0) fail_at(c.file, need(c, p, "count").line, "population.count must be positive");
    const std::string what = "population '" + name + "' params";
    const Node* par = p.get("params");
    if (model == "LIF" || model == "lif") {
        neuron::LIFOptions o;
        apply(c, par, {NRN_Q(LIF, v_rest), NRN_Q(LIF, v_thresh), NRN_Q(LIF, v_reset), NRN_Q(LIF, tau_m),
                       NRN_Q(LIF, tau_ref), NRN_Q(LIF, c_m), NRN_Q(LIF, i_bg)},
              what);
        auto* m = neuron::lif_create(n, o);
        neuron::lif_to_device(m, dev);
        return own_population(name, m, neuron::lif_as_module(m), n, neuron::lif_destroy, dev);
    }
    if (model == "AdEx" || model == "adex") {
        neuron::AdExOptions o;
        apply(c, par, {NRN_Q(AdEx, v_rest), NRN_Q(AdEx, v_thresh), NRN_Q(AdEx, v_reset), NRN_Q(AdEx, v_peak),
                       NRN_Q(AdEx, tau_m), NRN_Q(AdEx, tau_w), NRN_Q(AdEx, tau_ref), NRN_Q(AdEx, c_m),
                       NRN_Q(AdEx, g_l), NRN_Q(AdEx, a), NRN_Q(AdEx, b), NRN_Q(AdEx, delta_t), NRN_Q(AdEx, i_bg)},
              what);
        auto* m = neuron::adex_create(n, o);
        neuron::adex_to_device(m, dev);
        return own_population(name, m, neuron::adex_as_module(m), n, neuron::adex_destroy, dev);
    }
    if (model == "Izhikevich" || model == "izhikevich" || model == "Izh") {
        neuron::IzhikevichOptions o;
        apply(c, par, {NRN_Q(Izh, a), NRN_Q(Izh, b), NRN_Q(Izh, c), NRN_Q(Izh, d), NRN_Q(Izh, v_peak),
                       NRN_Q(Izh, v_init), NRN_Q(Izh, u_init)},
              what);
        auto* m = neuron::izh_create(n, o);
        neuron::izh_to_device(m, dev);
        return own_population(name, m, neuron::izh_as_module(m), n, neuron::izh_destroy, dev);
    }
    fail_at(c.file, need(c, p, "model").line, "unknown neuron model '" + model + "' (LIF, AdEx, Izhikevich)");
}

std::shared_ptr<Connection> make_connection(const Ctx& c, const Node& q, Region* r) {
    check_keys(c, q, {"source", "target", "topology", "probability", "allow_autapses", "sigma", "max_distance",
                      "min_probability", "weight", "block_size", "delay", "with_delays", "synapse", "synapse_params",
                      "plasticity", "plasticity_params"},
               "connection");
    auto find = [&](const char* key) {
        const Node& n = need(c, q, key);
        auto p = region_find_population(r, text(c, n, std::string("connection.") + key));
        if (!p) fail_at(c.file, n.line, std::string("connection.") + key + ": no population '" + n.text + "'");
        return p;
    };
    auto src = find("source");
    auto tgt = find("target");
    ConnectOptions co;
    if (const Node* n = q.get("weight")) co.weight_scale(quantity(c, *n, "connection.weight"));
    if (const Node* n = q.get("block_size")) co.block_size(integer(c, *n, "connection.block_size"));
    if (const Node* n = q.get("delay")) co.default_delay(quantity(c, *n, "connection.delay"));
    if (const Node* n = q.get("with_delays")) co.with_delays(boolean(c, *n, "connection.with_delays"));
    // synapse module (owned with the connection)
    std::function<void()> release;
    NrnModule syn{};
    const std::string sk = q.get("synapse") ? text(c, *q.get("synapse"), "connection.synapse") : "static";
    const Node* sp = q.get("synapse_params");
    const std::string what = "connection synapse_params";
    if (sk == "static") {
        StaticSynapseOptions o;
        apply(c, sp, {NRN_Q(Static, weight), NRN_Q(Static, delay)}, what);
        auto* s = synapse::static_synapse_create(tgt->n, o);
        syn = synapse::static_synapse_as_module(s);
        release = [s] { synapse::static_synapse_destroy(s); };
    } else if (sk == "exponential") {
        ExponentialSynapseOptions o;
        apply(c, sp, {NRN_Q(Exp, tau_decay), NRN_Q(Exp, weight), NRN_Q(Exp, delay)}, what);
        auto* s = synapse::exp_synapse_create(tgt->n, o);
        syn = synapse::exp_synapse_as_module(s);
        release = [s] { synapse::exp_synapse_destroy(s); };
    } else if (sk == "double_exponential") {
        DoubleExponentialSynapseOptions o;
        apply(c, sp, {NRN_Q(Dexp, tau_rise), NRN_Q(Dexp, tau_decay), NRN_Q(Dexp, weight), NRN_Q(Dexp, delay)}, what);
        auto* s = synapse::dexp_synapse_create(tgt->n, o);
        syn = synapse::dexp_synapse_as_module(s);
        release = [s] { synapse::dexp_synapse_destroy(s); };
    } else if (sk == "AMPA" || sk == "ampa") {
        AMPAOptions o;
        apply(c, sp, {NRN_Q(Ampa, tau_rise), NRN_Q(Ampa, tau_decay), NRN_Q(Ampa, e_rev), NRN_Q(Ampa, weight),
                      NRN_Q(Ampa, delay)},
              what);
        auto* s = synapse::ampa_create(tgt->n, o);
        syn = synapse::ampa_as_module(s);
        release = [s] { synapse::ampa_destroy(s); };
    } else {
        fail_at(c.file, q.get("synapse")->line,
                "unknown synapse '" + sk + "' (static, exponential, double_exponential, AMPA)");
    }
    // topology (only needed while connecting)
    const std::string topo = q.get("topology") ? text(c, *q.get("topology"), "connection.topology") : "random";
    std::shared_ptr<Connection> conn;
    if (topo == "random") {
        RandomTopologyOptions o;
        if (const Node* n = q.get("probability")) o.probability(quantity(c, *n, "connection.probability"));
        if (const Node* n = q.get("allow_autapses")) o.allow_autapses(boolean(c, *n, "connection.allow_autapses"));
        auto* t = random_topology_create(o);
        auto g = random_topology_as_generator(t);
        conn = connect(src, tgt, &g, syn, co);
        random_topology_destroy(t);
    } else if (topo == "distance_dependent") {
        DistanceDependentOptions o;
        if (const Node* n = q.get("sigma")) o.sigma(quantity(c, *n, "connection.sigma"));
        if (const Node* n = q.get("max_distance")) o.max_distance(quantity(c, *n, "connection.max_distance"));
        if (const Node* n = q.get("min_probability")) o.min_probability(quantity(c, *n, "connection.min_probability"));
        auto* t = distance_dep_topology_create(o);
        auto g = distance_dep_topology_as_generator(t);
        conn = connect(src, tgt, &g, syn, co);
        distance_dep_topology_destroy(t);
    } else {
        fail_at(c.file, q.get("topology")->line, "unknown topology '" + topo + "' (random, distance_dependent)");
    }
    if (const Node* pl = q.get("plasticity")) {
        const std::string kind = text(c, *pl, "connection.plasticity");
        if (kind != "stdp" && kind != "STDP") fail_at(c.file, pl->line, "unknown plasticity '" + kind + "' (stdp)");
        STDPOptions o;
        apply(c, q.get("plasticity_params"),
              {NRN_Q(STDP, tau_plus), NRN_Q(STDP, tau_minus), NRN_Q(STDP, a_plus), NRN_Q(STDP, a_minus),
               NRN_Q(STDP, w_max), NRN_Q(STDP, w_min), NRN_Q(STDP, learning_rate)},
              "connection plasticity_params");
        auto* st = stdp_create(o);
        connection_attach(conn.get(), stdp_as_rule(st));
        auto prev = release;
        release = [prev, st] {
            prev();
            stdp_destroy(st);
        };
    }
    auto h = std::make_shared<ConnHolder>();
    h->conn = conn;
    h->release = release;
    return std::shared_ptr<Connection>(h, conn.get());
}

Node read_file(const std::string& path) {
    std::ifstream f(path);
    if (!f) throw std::runtime_error("nrn::config: cannot open '" + path + "'");
    std::stringstream ss;
    ss << f.rdbuf();
    Node root = Reader(path, ss.str()).parse();
    if (root.kind != Node::Map) fail_at(path, root.line, "the file must hold a mapping");
    return root;
}

Region* build_region(const Ctx& c, const Node& root) {
    const Node* sim = root.get("simulation");
    const torch::Device dev = device_of(c, sim);
    if (const Node* s = root.get("seed")) torch::manual_seed(static_cast<uint64_t>(integer(c, *s, "seed")));
    const std::string name = root.get("name") ? text(c, *root.get("name"), "name") : "region";
    std::unique_ptr<Region> r(region_create(name));
    const Node* pops = root.get("populations");
    if (!pops || pops->kind != Node::Seq || pops->seq.empty())
        fail_at(c.file, root.line, "'populations' must be a non-empty sequence");
    for (const auto& p : pops->seq) {
        if (p.kind != Node::Map) fail_at(c.file, p.line, "a population must be a mapping");
        auto pop = make_population(c, p, dev);
        if (region_find_population(r.get(), pop->name))
            fail_at(c.file, p.line, "duplicate population '" + pop->name + "'");
        region_add_population(r.get(), pop);
    }
    if (const Node* conns = root.get("connections")) {
        if (conns->kind != Node::Seq) fail_at(c.file, conns->line, "'connections' must be a sequence");
        for (const auto& q : conns->seq) {
            if (q.kind != Node::Map) fail_at(c.file, q.line, "a connection must be a mapping");
            region_add_connection(r.get(), make_connection(c, q, r.get()));
        }
    }
    return r.release();
}

}  // namespace

Region* load_region(const std::string& path) {
    const Node root = read_file(path);
    Ctx c{path};
    check_keys(c, root, {"name", "seed", "simulation", "populations", "connections", "record"}, "top level");
    return build_region(c, root);
}

Simulation* load(const std::string& path) {
    const Node root = read_file(path);
    Ctx c{path};
    check_keys(c, root, {"name", "seed", "simulation", "populations", "connections", "record"}, "top level");
    Region* r = build_region(c, root);
    SimulationOptions o;
    o.device(device_of(c, root.get("simulation")));
    try {
        const Node* s = root.get("simulation");
        const std::string what = "simulation";
        apply(c, s,
              {NRN_Q(Sim, dt_fast), NRN_Q(Sim, dt_slow), NRN_Q(Sim, dt_structural), NRN_Q(Sim, duration),
               {"device", [](const Node&) {}},
               {"use_cuda_graphs", [&](const Node& n) { o.use_cuda_graphs(boolean(c, n, "simulation.use_cuda_graphs")); }},
               {"max_delay_steps", [&](const Node& n) { o.max_delay_steps(integer(c, n, "simulation.max_delay_steps")); }}},
              what);
        // The Simulation refers to the Region but does not own it (as with
        // sim_create); a loaded Simulation keeps its Region for the process.
        Simulation* sim = sim_create(r, o);
        if (const Node* rec = root.get("record")) {
            if (rec->kind != Node::Seq) fail_at(c.file, rec->line, "'record' must be a sequence");
            for (const auto& e : rec->seq) {
                check_keys(c, e, {"population", "variables"}, "record");
                const Node& pn = need(c, e, "population");
                auto pop = region_find_population(r, text(c, pn, "record.population"));
                if (!pop) fail_at(c.file, pn.line, "record: no population '" + pn.text + "'");
                std::vector<std::string> vars;
                const Node& vn = need(c, e, "variables");
                if (vn.kind != Node::Seq) fail_at(c.file, vn.line, "record.variables must be a sequence");
                for (const auto& v : vn.seq) vars.push_back(text(c, v, "record.variables"));
                sim_record(sim, pop, vars);
            }
        }
        return sim;
    } catch (...) {
        region_destroy(r);
        throw;
    }
}

#undef NRN_Q

}  // namespace config
}  // namespace nrn
