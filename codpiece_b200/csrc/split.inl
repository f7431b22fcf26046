// split.inl — tensor-parallel partition rules (host code).
//
// Restates crates/codpiece-model/src/split.rs: classify() (split.rs:73-196),
// rotation() (201-217), granularity() (231-283) and split_state() (298-333),
// and the fallback behaviour of the C callback in meta.rs:47-121 (never
// fails; anything unexpected degrades to MIRRORED). The rules are the
// reference's (a wrong split is silently wrong, so they must agree exactly);
// the code is this project's.
//
// One deliberate extension: cpq_hparams.q_has_gate. The reference's attn_q is
// 2*n_head*head_k rows (Q and a gate interleaved per head), so its split
// granularity is twice the attention output's (split.rs:268-269). A plain q
// projection of n_head*head_k rows (the benchmark's 27B-shaped stack) must
// split at the attention output's granularity, or q's output slice and
// attn_output's input slice stop lining up.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace cpq {
namespace split {

enum Axis { kAxis0 = CPQ_SPLIT_AXIS_0, kAxis1 = CPQ_SPLIT_AXIS_1, kAxis2 = CPQ_SPLIT_AXIS_2,
            kMirrored = CPQ_SPLIT_MIRRORED, kPartial = CPQ_SPLIT_PARTIAL };

struct Seg {
    int64_t size;
    uint32_t rep;
};

struct Split {
    Axis axis;
    std::vector<Seg> segments;  // empty: one segment covering the whole axis
};

static bool starts_with(const std::string &s, const char *p) { return s.rfind(p, 0) == 0; }

static bool is_recurrent(const cpq_hparams &hp, int64_t il) {
    return hp.full_attn_interval > 0 && (il + 1) % hp.full_attn_interval != 0;
}

// "blk.<N>.<rest>" -> (N, rest)
static bool layer_of(const std::string &name, int64_t *il, std::string *suffix) {
    if (!starts_with(name, "blk.")) return false;
    const std::string rest = name.substr(4);
    const size_t dot = rest.find('.');
    if (dot == std::string::npos || dot == 0) return false;
    const std::string num = rest.substr(0, dot);
    for (char c : num)
        if (c < '0' || c > '9') return false;
    *il = std::strtoll(num.c_str(), nullptr, 10);
    *suffix = rest.substr(dot + 1);
    return true;
}

// "cache_<kind>_l<N>" -> (kind, N); kind is the text before the first "_l"
static bool cache_of(const std::string &name, std::string *kind, int64_t *il) {
    if (!starts_with(name, "cache_")) return false;
    const std::string rest = name.substr(6);
    const size_t p = rest.find("_l");
    *kind = p == std::string::npos ? rest : rest.substr(0, p);
    if (p == std::string::npos) return false;
    const std::string num = rest.substr(p + 2);
    if (num.empty()) return false;
    for (char c : num)
        if (c < '0' || c > '9') return false;
    *il = std::strtoll(num.c_str(), nullptr, 10);
    return true;
}

static Split classify(const std::string &name, const cpq_hparams &hp) {
    const Split mirrored{kMirrored, {}};
    if (starts_with(name, "dflash.")) return mirrored;  // drafter: replicated wholesale
    const uint32_t head_ratio = hp.n_k_heads > 0 ? uint32_t(hp.n_v_heads / hp.n_k_heads) : 1;
    const int64_t key_dim = hp.d_state * hp.n_k_heads;

    if (starts_with(name, "cache_")) {
        std::string kind;
        int64_t il;
        const std::string rest = name.substr(6);
        const size_t p = rest.find("_l");
        kind = p == std::string::npos ? rest : rest.substr(0, p);
        (void)il;
        if (kind == "k" || kind == "v") return {kAxis0, {}};
        if (kind == "conv") return {kAxis1, {{key_dim, 2 + head_ratio}}};
        if (kind == "gdn") return {kAxis2, {{hp.n_k_heads, head_ratio}}};
        return mirrored;
    }

    int64_t il;
    std::string s;
    if (!layer_of(name, &il, &s)) {
        if (name == "output.weight") return hp.split_output ? Split{kAxis1, {}} : mirrored;
        if (name == "output.bias") return {kAxis0, {}};
        return mirrored;
    }
    if (s == "attn_qkv.weight") return {kAxis1, {{key_dim, 2 + head_ratio}}};
    if (s == "attn_q.weight" || s == "attn_k.weight" || s == "attn_v.weight") return {kAxis1, {}};
    if (s == "attn_q.bias" || s == "attn_k.bias" || s == "attn_v.bias" || s == "attn_qkv.bias") return {kAxis0, {}};
    if (s == "attn_q_norm.weight" || s == "attn_k_norm.weight") return mirrored;
    if (s == "attn_output.weight") return {kAxis0, {}};
    if (s == "attn_output.bias") return mirrored;
    if (s == "attn_gate.weight") return {kAxis1, {{key_dim, head_ratio}}};
    if (s == "ssm_dt.bias" || s == "ssm_a") return {kAxis0, {{hp.n_k_heads, head_ratio}}};
    if (s == "ssm_alpha.weight" || s == "ssm_beta.weight") return {kAxis1, {{hp.n_k_heads, head_ratio}}};
    if (s == "ssm_conv1d.weight") return {kAxis1, {{key_dim, 2 + head_ratio}}};
    if (s == "ssm_out.weight") return {kAxis0, {{key_dim, head_ratio}}};
    if (s == "ssm_norm.weight") return mirrored;
    if (s == "ffn_up.weight" || s == "ffn_gate.weight") return {kAxis1, {}};
    if (s == "ffn_up.bias" || s == "ffn_gate.bias") return {kAxis0, {}};
    if (s == "ffn_down.weight") return {kAxis0, {}};
    if (s == "ffn_down.bias") return mirrored;
    return mirrored;
}

// Leftover rows alternate between devices layer by layer, counting only
// previous layers of the same kind (recurrent vs attention).
static int64_t rotation(const std::string &name, const cpq_hparams &hp, int n_devices) {
    int64_t il = -1;
    std::string s, kind;
    if (!layer_of(name, &il, &s)) {
        if (!cache_of(name, &kind, &il)) il = -1;
    }
    if (il < 0) return hp.n_layer % n_devices;
    const bool rec = is_recurrent(hp, il);
    int64_t same = 0;
    for (int64_t p = 0; p < il; p++)
        if (is_recurrent(hp, p) == rec) same++;
    return same % n_devices;
}

static int64_t gcd64(int64_t a, int64_t b) { return b == 0 ? (a < 0 ? -a : a) : gcd64(b, a % b); }
static int64_t lcm64(int64_t a, int64_t b) {
    if (a == 0 || b == 0) return 0;
    const int64_t r = a / gcd64(a, b) * b;
    return r < 0 ? -r : r;
}

static int64_t granularity(const std::string &name, const cpq_hparams &hp, int64_t blck, int n_devices) {
    int64_t il;
    std::string s;
    if (!layer_of(name, &il, &s)) {
        std::string kind;
        if (!cache_of(name, &kind, &il)) return 1;
        s = kind;
    }
    if (is_recurrent(hp, il)) {
        const int64_t head_dim = hp.d_state;
        const int64_t g_qkv = lcm64(lcm64(blck, 128), head_dim);
        if (s == "attn_qkv.weight" || s == "attn_gate.weight" || s == "ssm_conv1d.weight" || s == "ssm_out.weight" ||
            s == "conv")
            return g_qkv;
        if (s == "ssm_dt.bias" || s == "ssm_a" || s == "ssm_alpha.weight" || s == "ssm_beta.weight" || s == "gdn")
            return head_dim ? g_qkv / head_dim : 1;
    } else {
        const int64_t n_gqa = hp.n_head_kv ? hp.n_head / hp.n_head_kv : 1;
        const int64_t n_embd_q = n_gqa * hp.head_k;
        int64_t blck_perf = blck;
        while (blck_perf < 128 && blck_perf * n_devices < n_embd_q) blck_perf *= 2;
        const int64_t g_q = lcm64(n_embd_q, blck_perf);
        if (s == "attn_q.weight" || s == "attn_q.bias")
            return hp.q_has_gate ? lcm64(2 * n_embd_q, blck_perf) : g_q;
        if (s == "attn_output.weight") return g_q;
        if (s == "attn_k.weight" || s == "attn_v.weight" || s == "attn_k.bias" || s == "attn_v.bias" || s == "k" ||
            s == "v")
            return n_gqa ? g_q / n_gqa : 1;
    }
    if (s == "ffn_up.weight" || s == "ffn_gate.weight" || s == "ffn_down.weight" || s == "ffn_up.bias" ||
        s == "ffn_gate.bias")
        return lcm64(blck, 128);
    return 1;
}

static cpq_split_state mirrored_state() {
    cpq_split_state st;
    std::memset(&st, 0, sizeof st);
    st.axis = CPQ_SPLIT_MIRRORED;
    st.n_segments = 1;
    st.nr[0] = 1;
    return st;
}

static cpq_split_state split_state(const std::string &name, const cpq_hparams &hp, int64_t extent, int64_t blck,
                                   int n_devices) {
    const Split sp = classify(name, hp);
    cpq_split_state st = mirrored_state();
    st.axis = sp.axis;
    if (sp.axis != kAxis0 && sp.axis != kAxis1 && sp.axis != kAxis2) return st;
    std::vector<Seg> segs = sp.segments.empty() ? std::vector<Seg>{{extent, 1}} : sp.segments;
    if (segs.size() > 16 || segs.size() * size_t(n_devices) > 256) return mirrored_state();
    const int64_t g = std::max<int64_t>(granularity(name, hp, blck, n_devices), 1);
    const int64_t rot = rotation(name, hp, n_devices);
    for (size_t is = 0; is < segs.size(); is++) {
        const int64_t ne_s = segs[is].size;
        int64_t low = 0;
        for (int j = 0; j < n_devices - 1; j++) {
            int64_t high = ne_s * (j + 1) / n_devices;
            high -= high % g;
            st.ne[is * n_devices + (j + rot) % n_devices] = high - low;
            low = high;
        }
        st.ne[is * n_devices + (n_devices - 1 + rot) % n_devices] = ne_s - low;
        st.nr[is] = segs[is].rep;
    }
    st.n_segments = uint32_t(segs.size());
    return st;
}

}  // namespace split
}  // namespace cpq

extern "C" cpq_split_state cpq_tp_split_state(const char *name, const cpq_hparams *hp, int64_t extent, int64_t blck,
                                              int n_devices) {
    if (!name || !hp || n_devices < 1 || n_devices > 256 || extent < 0) return cpq::split::mirrored_state();
    try {
        return cpq::split::split_state(std::string(name), *hp, extent, blck, n_devices);
    } catch (...) {
        return cpq::split::mirrored_state();
    }
}
