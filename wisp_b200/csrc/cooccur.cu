// Cross-layer expert co-activation table and the prefetch predictor, native
// (host C++).  The same table and arithmetic as the reference's
// CooccurTable / predict_layer (src/wisp/oracle/cooccur.py:44-292), which the
// paged forward's post-forward block drives once per layer of a decode step
// (src/wisp/integrations/vllm/fused_moe.py:1170-1233): there a prediction
// walks every earlier layer's experts in Python, milliseconds per layer.
//
//   observe_step    for one decode step's {layer: experts} (layers in the
//                   given order, empty ones skipped): every (L, e) marginal
//                   +1; for every source (L_src, e_src) its entry is created
//                   (even when no later layer follows) and every later layer's
//                   experts e_dst get +1 in row (L_src, e_src) -> L_dst;
//   predict         score[e_dst] = sum over the seen sources, in the given
//                   layer order and list order, of
//                   w * count / denom, w = decay^(target - L_src - 1),
//                   denom = the source's marginal when normalising (1 when it
//                   is 0 or normalisation is off), evaluated as (w * count) /
//                   denom in double, left to right -- the reference's
//                   expression -- then the top k by (score descending, id
//                   ascending).
// Sources, rows and entries keep their first-seen order, so the export (the
// reference's JSON schema: pairs [L_src, e_src, L_dst, e_dst, n] with n > 0,
// marginals [L, e, n]) lists them in the reference's dict order.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <new>
#include <unordered_map>
#include <vector>

#include "common.cuh"

struct wisp_cooccur {
    // One row (L_src, e_src) -> L_dst: entries in first-seen order (ids and
    // counts apart, so a prediction streams them), and the same entries' indices
    // sorted by id for the updates of observe_step (binary search).
    struct Row {
        int32_t l_dst;
        std::vector<int32_t> ids;
        std::vector<int64_t> n;
        std::vector<int32_t> by_id;  // indices into ids, ascending by id
    };
    struct Source {
        int32_t l, e;
        std::vector<Row> rows;         // first-seen order of L_dst
        std::vector<int32_t> row_of;   // L_dst -> index + 1 into rows (0: none)
    };
    std::vector<Source> sources;                          // first-seen order of (L_src, e_src)
    std::unordered_map<int64_t, int32_t> source_of;       // (L, e) key -> index in sources
    std::vector<std::pair<int64_t, int64_t>> marginals;   // ((L, e) key, n), first-seen order
    std::unordered_map<int64_t, int32_t> marginal_of;
    int64_t steps = 0;

    static int64_t key(int32_t l, int32_t e) { return ((int64_t)l << 32) | (uint32_t)e; }

    int32_t source(int32_t l, int32_t e) {
        const int64_t k = key(l, e);
        auto it = source_of.find(k);
        if (it != source_of.end()) return it->second;
        const int32_t i = (int32_t)sources.size();
        source_of.emplace(k, i);
        sources.push_back(Source{l, e, {}, {}});
        return i;
    }
    static Row &row(Source &s, int32_t l_dst) {
        if (l_dst >= 0 && (size_t)l_dst < s.row_of.size() && s.row_of[l_dst]) return s.rows[s.row_of[l_dst] - 1];
        if (l_dst >= 0) {
            if ((size_t)l_dst >= s.row_of.size()) s.row_of.resize((size_t)l_dst + 1, 0);
            s.row_of[l_dst] = (int32_t)s.rows.size() + 1;
        } else {
            for (Row &r : s.rows)  // negative layer ids: no index, a scan
                if (r.l_dst == l_dst) return r;
        }
        s.rows.push_back(Row{l_dst, {}, {}, {}});
        return s.rows.back();
    }
    static const Row *find_row(const Source &s, int32_t l_dst) {
        if (l_dst >= 0) {
            if ((size_t)l_dst < s.row_of.size() && s.row_of[l_dst]) return &s.rows[s.row_of[l_dst] - 1];
            return nullptr;
        }
        for (const Row &r : s.rows)
            if (r.l_dst == l_dst) return &r;
        return nullptr;
    }
    static int64_t &entry(Row &r, int32_t e_dst) {
        auto it = std::lower_bound(r.by_id.begin(), r.by_id.end(), e_dst,
                                   [&](int32_t idx, int32_t v) { return r.ids[idx] < v; });
        if (it != r.by_id.end() && r.ids[*it] == e_dst) return r.n[*it];
        const int32_t idx = (int32_t)r.ids.size();
        r.ids.push_back(e_dst);
        r.n.push_back(0);
        r.by_id.insert(it, idx);
        return r.n.back();
    }
    int64_t &marginal(int32_t l, int32_t e) {
        const int64_t k = key(l, e);
        auto it = marginal_of.find(k);
        if (it != marginal_of.end()) return marginals[it->second].second;
        marginal_of.emplace(k, (int32_t)marginals.size());
        marginals.emplace_back(k, 0);
        return marginals.back().second;
    }
    int64_t marginal_or_zero(int32_t l, int32_t e) const {
        auto it = marginal_of.find(key(l, e));
        return it == marginal_of.end() ? 0 : marginals[it->second].second;
    }
    const Source *find_source(int32_t l, int32_t e) const {
        auto it = source_of.find(key(l, e));
        return it == source_of.end() ? nullptr : &sources[it->second];
    }
};

using wisp::set_error;

namespace {
bool bad_csr(int32_t n, const int32_t *layers, const int32_t *offsets, const int32_t *experts) {
    if (n < 0 || (n > 0 && (!layers || !offsets))) return true;
    if (n > 0 && offsets[0] != 0) return true;
    for (int32_t i = 0; i < n; ++i)
        if (offsets[i + 1] < offsets[i]) return true;
    return n > 0 && offsets[n] > 0 && !experts;
}
}  // namespace

extern "C" {

int wisp_cooccur_create(wisp_cooccur **out) {
    if (!out) return set_error("wisp_cooccur_create: NULL out"), WISP_ERR_INVALID;
    *out = new (std::nothrow) wisp_cooccur();
    return *out ? WISP_OK : (set_error("wisp_cooccur_create: out of host memory"), WISP_ERR_NOMEM);
}

int wisp_cooccur_destroy(wisp_cooccur *t) {
    delete t;
    return WISP_OK;
}

int wisp_cooccur_observe_step(wisp_cooccur *t, int32_t n_layers, const int32_t *layers, const int32_t *offsets,
                              const int32_t *experts) {
    if (!t || bad_csr(n_layers, layers, offsets, experts))
        return set_error("wisp_cooccur_observe_step: bad arguments"), WISP_ERR_INVALID;
    std::vector<int32_t> live;  // layers with experts, in the given order
    for (int32_t i = 0; i < n_layers; ++i)
        if (offsets[i + 1] > offsets[i]) live.push_back(i);
    for (int32_t i : live)
        for (int32_t j = offsets[i]; j < offsets[i + 1]; ++j) t->marginal(layers[i], experts[j]) += 1;
    for (int32_t i : live) {
        for (int32_t j = offsets[i]; j < offsets[i + 1]; ++j) {
            // the source's entry exists from its first observation on (even with no later layer)
            const int32_t si = t->source(layers[i], experts[j]);
            for (int32_t d : live) {
                if (layers[d] <= layers[i]) continue;
                wisp_cooccur::Row &r = wisp_cooccur::row(t->sources[si], layers[d]);
                for (int32_t q = offsets[d]; q < offsets[d + 1]; ++q) wisp_cooccur::entry(r, experts[q]) += 1;
            }
        }
    }
    t->steps += 1;
    return WISP_OK;
}

int wisp_cooccur_predict(const wisp_cooccur *t, int32_t n_seen, const int32_t *layers, const int32_t *offsets,
                         const int32_t *experts, int32_t target_layer, int32_t k, int32_t normalize, double decay,
                         int32_t only_prev_layer, int32_t *out_ids, int32_t *n_out) {
    if (!t || !n_out || k < 0 || (k > 0 && !out_ids) || bad_csr(n_seen, layers, offsets, experts))
        return set_error("wisp_cooccur_predict: bad arguments"), WISP_ERR_INVALID;
    // dense scores over the expert ids seen (a flag marks the scored ones)
    std::vector<double> score;
    std::vector<char> scored;
    std::vector<int32_t> order;  // experts with a score (any order: the ranking breaks ties by id)
    for (int32_t i = 0; i < n_seen; ++i) {
        const int32_t l_src = layers[i];
        if (l_src >= target_layer || (only_prev_layer && l_src != target_layer - 1)) continue;
        const double w = std::pow(decay, (double)(target_layer - l_src - 1));
        for (int32_t j = offsets[i]; j < offsets[i + 1]; ++j) {
            const wisp_cooccur::Source *s = t->find_source(l_src, experts[j]);
            if (!s) continue;
            const wisp_cooccur::Row *r = wisp_cooccur::find_row(*s, target_layer);
            if (!r || r->ids.empty()) continue;
            const int64_t total = normalize ? t->marginal_or_zero(l_src, experts[j]) : 1;
            const double denom = (normalize && total > 0) ? (double)total : 1.0;
            const size_t ne = r->ids.size();
            for (size_t q = 0; q < ne; ++q) {
                const double add = w * (double)r->n[q] / denom;
                const int32_t id = r->ids[q];
                const size_t e = (size_t)(uint32_t)id;
                if (e >= score.size()) {
                    score.resize(e + 1, 0.0);
                    scored.resize(e + 1, 0);
                }
                if (!scored[e]) {
                    scored[e] = 1;
                    score[e] = 0.0 + add;
                    order.push_back(id);
                } else {
                    score[e] = score[e] + add;
                }
            }
        }
    }
    std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
        const double sa = score[(uint32_t)a], sb = score[(uint32_t)b];
        return sa != sb ? sa > sb : a < b;
    });
    const int32_t n = std::min<int32_t>(k, (int32_t)order.size());
    for (int32_t i = 0; i < n; ++i) out_ids[i] = order[i];
    *n_out = n;
    return WISP_OK;
}

int wisp_cooccur_set_pair(wisp_cooccur *t, int32_t l_src, int32_t e_src, int32_t l_dst, int32_t e_dst, int64_t n) {
    if (!t) return set_error("wisp_cooccur_set_pair: NULL table"), WISP_ERR_INVALID;
    const int32_t si = t->source(l_src, e_src);
    wisp_cooccur::entry(wisp_cooccur::row(t->sources[si], l_dst), e_dst) = n;
    return WISP_OK;
}

int wisp_cooccur_set_marginal(wisp_cooccur *t, int32_t l, int32_t e, int64_t n) {
    if (!t) return set_error("wisp_cooccur_set_marginal: NULL table"), WISP_ERR_INVALID;
    t->marginal(l, e) = n;
    return WISP_OK;
}

int wisp_cooccur_set_steps(wisp_cooccur *t, int64_t steps) {
    if (!t || steps < 0) return set_error("wisp_cooccur_set_steps: bad arguments"), WISP_ERR_INVALID;
    t->steps = steps;
    return WISP_OK;
}

int wisp_cooccur_sizes(const wisp_cooccur *t, int64_t *n_sources, int64_t *n_pairs, int64_t *n_marginals,
                       int64_t *steps) {
    if (!t) return set_error("wisp_cooccur_sizes: NULL table"), WISP_ERR_INVALID;
    int64_t pairs = 0;
    for (const auto &s : t->sources)
        for (const auto &r : s.rows) pairs += (int64_t)r.ids.size();
    if (n_sources) *n_sources = (int64_t)t->sources.size();
    if (n_pairs) *n_pairs = pairs;
    if (n_marginals) *n_marginals = (int64_t)t->marginals.size();
    if (steps) *steps = t->steps;
    return WISP_OK;
}

int wisp_cooccur_export(const wisp_cooccur *t, int64_t *pairs, int64_t max_pairs, int64_t *n_pairs_out,
                        int64_t *marginals, int64_t max_marginals, int64_t *n_marginals_out) {
    if (!t || !n_pairs_out || !n_marginals_out || (max_pairs > 0 && !pairs) || (max_marginals > 0 && !marginals))
        return set_error("wisp_cooccur_export: bad arguments"), WISP_ERR_INVALID;
    int64_t np = 0, nm = 0;
    for (const auto &s : t->sources)
        for (const auto &r : s.rows)
            for (size_t q = 0; q < r.ids.size(); ++q) {
                if (r.n[q] <= 0) continue;
                if (np < max_pairs) {
                    int64_t *p = pairs + 5 * np;
                    p[0] = s.l;
                    p[1] = s.e;
                    p[2] = r.l_dst;
                    p[3] = r.ids[q];
                    p[4] = r.n[q];
                }
                ++np;
            }
    for (const auto &m : t->marginals) {
        if (m.second <= 0) continue;
        if (nm < max_marginals) {
            int64_t *p = marginals + 3 * nm;
            p[0] = (int32_t)(m.first >> 32);
            p[1] = (int32_t)(uint32_t)(m.first & 0xffffffffu);
            p[2] = m.second;
        }
        ++nm;
    }
    *n_pairs_out = np;
    *n_marginals_out = nm;
    return WISP_OK;
}

}  // extern "C"
