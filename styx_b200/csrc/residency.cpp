// residency.cpp -- host-side expert residency planning (include/styx_residency.h).
//
// Restates MoeModel's placement decisions (crates/model/src/moe.rs): the
// auto budget (:741-753), popularity pinning (:776-813, hot_order :825-835),
// the per-layer remap / hot mask / slot tables (:984-995), online repinning
// (:1450-1505), the HUD hot/cold counts (:1512-1521) and the prefetch plan
// (:2169-2213).  Pure host code over plain arrays; the decisions are applied
// by the caller through the styx_moe.h copy and upload entry points.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/styx_residency.h"
#include "kernels.h"

struct styx_residency {
    int n_layers = 0, n_expert = 0, k = 0;
    uint64_t cost = 0;
    // per layer: remap (expert -> hot slot or SKIP), hot slot -> expert, hits
    std::vector<std::vector<uint32_t>> remap;
    std::vector<std::vector<uint32_t>> slot_experts;
    std::vector<std::vector<uint64_t>> hits;
};

namespace {

int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return styx::set_error(code, buf);
}

#define RNEED(cond, ...)                                                                           \
    do {                                                                                           \
        if (!(cond)) return fail(STYX_EINVAL, __VA_ARGS__);                                        \
    } while (0)

// routed expert id of (layer, slot) in an ids buffer, -1 if out of range
inline int routed(const styx_residency &r, const int32_t *ids, int layer, int s) {
    const int32_t e = ids[static_cast<size_t>(layer) * STYX_IDS_PER_LAYER + s];
    return (e >= 0 && e < r.n_expert) ? e : -1;
}

// Entries are (hits, layer, expert) in input order.  Ranked by hits, hottest
// first, equal hits in input order; each pins while the budget covers one
// more expert's cost (moe.rs:793-810), then the hot slots of every layer hold
// its pinned experts in ascending id order (moe.rs:825-835, 984-995).
int pin_entries(styx_residency *r, std::vector<std::pair<uint64_t, std::pair<int, int>>> &entries,
                uint64_t budget, int *n_pinned) {
    std::stable_sort(entries.begin(), entries.end(),
                     [](const auto &a, const auto &b) { return a.first > b.first; });
    std::vector<std::vector<uint8_t>> hot(r->n_layers, std::vector<uint8_t>(r->n_expert, 0));
    uint64_t left = budget;
    int pinned = 0;
    for (const auto &en : entries) {
        if (left < r->cost) break;
        left -= r->cost;
        const int l = en.second.first, e = en.second.second;
        if (!hot[l][e]) pinned++;
        hot[l][e] = 1;   // the reference inserts into a set: a repeated entry costs again, pins once
    }
    for (int l = 0; l < r->n_layers; l++) {
        r->remap[l].assign(r->n_expert, STYX_SKIP);
        r->slot_experts[l].clear();
        for (int e = 0; e < r->n_expert; e++)
            if (hot[l][e]) {
                r->remap[l][e] = static_cast<uint32_t>(r->slot_experts[l].size());
                r->slot_experts[l].push_back(static_cast<uint32_t>(e));
            }
        r->hits[l].assign(r->n_expert, 0);
    }
    if (n_pinned) *n_pinned = pinned;
    return STYX_OK;
}

// one unsigned decimal field of a CSV line, as Rust's unsigned str::parse:
// ASCII digits with at most one leading '+', no overflow
bool parse_u64(const std::string &s0, uint64_t &v) {
    const std::string s = (!s0.empty() && s0[0] == '+') ? s0.substr(1) : s0;
    if (s.empty()) return false;
    v = 0;
    for (char c : s) {
        if (c < '0' || c > '9') return false;
        const uint64_t d = static_cast<uint64_t>(c - '0');
        if (v > (UINT64_MAX - d) / 10) return false;
        v = v * 10 + d;
    }
    return true;
}

}  // namespace

extern "C" {

uint64_t styx_expert_budget(uint64_t device_vram, uint64_t headroom_bytes, uint64_t pinned_bytes,
                            uint64_t kv_max_bytes, uint64_t arena_bytes, int has_explicit,
                            uint64_t explicit_bytes, int all_vram) {
    if (all_vram) return UINT64_MAX;
    if (has_explicit) return explicit_bytes;
    // saturating sum of the reservations, then saturating difference
    uint64_t res = 0;
    for (uint64_t v : {headroom_bytes, pinned_bytes, kv_max_bytes, arena_bytes})
        res = (res > UINT64_MAX - v) ? UINT64_MAX : res + v;
    return device_vram > res ? device_vram - res : 0;
}

uint64_t styx_arena_bytes(int n_layers, int k, const uint64_t max_slab[3]) {
    if (n_layers <= 0 || k <= 0 || !max_slab) return 0;
    return static_cast<uint64_t>(n_layers) * static_cast<uint64_t>(k) * (max_slab[0] + max_slab[1] + max_slab[2]);
}

int styx_residency_create(int n_layers, int n_expert, int k, uint64_t cost_per_expert, styx_residency **out) {
    RNEED(out, "null out");
    RNEED(n_layers > 0 && n_expert > 0 && n_expert <= STYX_MAX_EXPERTS, "bad n_layers %d / n_expert %d", n_layers,
          n_expert);
    RNEED(k > 0 && k <= STYX_MAX_TOPK && k <= n_expert, "bad k %d", k);
    RNEED(cost_per_expert > 0, "cost_per_expert must be positive");
    styx_residency *r = new (std::nothrow) styx_residency;
    if (!r) return fail(STYX_ENOMEM, "out of host memory");
    r->n_layers = n_layers;
    r->n_expert = n_expert;
    r->k = k;
    r->cost = cost_per_expert;
    r->remap.assign(n_layers, std::vector<uint32_t>(n_expert, STYX_SKIP));
    r->slot_experts.assign(n_layers, {});
    r->hits.assign(n_layers, std::vector<uint64_t>(n_expert, 0));
    *out = r;
    return STYX_OK;
}

void styx_residency_destroy(styx_residency *r) { delete r; }

int styx_residency_pin(styx_residency *r, const int32_t *layer, const int32_t *expert, const uint64_t *hits, int n,
                       uint64_t budget, int *n_pinned) {
    RNEED(r, "null residency");
    RNEED(n >= 0 && (n == 0 || (layer && expert && hits)), "bad entries");
    std::vector<std::pair<uint64_t, std::pair<int, int>>> entries;
    entries.reserve(static_cast<size_t>(n));
    for (int i = 0; i < n; i++) {
        RNEED(layer[i] >= 0 && layer[i] < r->n_layers && expert[i] >= 0 && expert[i] < r->n_expert,
              "entry %d: (layer %d, expert %d) out of range", i, layer[i], expert[i]);
        entries.push_back({hits[i], {layer[i], expert[i]}});
    }
    return pin_entries(r, entries, budget, n_pinned);
}

int styx_residency_pin_csv(styx_residency *r, const char *text, size_t len, uint64_t budget, int *n_pinned) {
    RNEED(r, "null residency");
    RNEED(text || len == 0, "null text");
    std::vector<std::pair<uint64_t, std::pair<int, int>>> entries;
    size_t pos = 0;
    bool header = true;   // .lines().skip(1)
    while (pos < len) {
        size_t end = pos;
        while (end < len && text[end] != '\n') end++;
        std::string line(text + pos, end - pos);
        pos = end + 1;
        if (!line.empty() && line.back() == '\r') line.pop_back();   // str::lines strips "\r\n"
        if (header) {
            header = false;
            continue;
        }
        // split(','): the first three fields must parse; extra fields are ignored
        std::vector<std::string> f;
        size_t a = 0;
        for (size_t i = 0; i <= line.size(); i++)
            if (i == line.size() || line[i] == ',') {
                f.push_back(line.substr(a, i - a));
                a = i + 1;
            }
        uint64_t l, e, h;
        if (f.size() < 3 || !parse_u64(f[0], l) || !parse_u64(f[1], e) || !parse_u64(f[2], h)) continue;
        if (e > UINT32_MAX) continue;   // the reference parses the expert as u32
        RNEED(l < static_cast<uint64_t>(r->n_layers) && e < static_cast<uint64_t>(r->n_expert),
              "histogram line (layer %llu, expert %llu) out of range", (unsigned long long)l, (unsigned long long)e);
        entries.push_back({h, {static_cast<int>(l), static_cast<int>(e)}});
    }
    return pin_entries(r, entries, budget, n_pinned);
}

int styx_residency_layer(const styx_residency *r, int layer, uint32_t *remap, uint32_t *slot_experts, int *n_slots) {
    RNEED(r, "null residency");
    RNEED(layer >= 0 && layer < r->n_layers, "layer %d out of range", layer);
    if (remap) std::memcpy(remap, r->remap[layer].data(), r->remap[layer].size() * 4);
    if (slot_experts && !r->slot_experts[layer].empty())
        std::memcpy(slot_experts, r->slot_experts[layer].data(), r->slot_experts[layer].size() * 4);
    if (n_slots) *n_slots = static_cast<int>(r->slot_experts[layer].size());
    return STYX_OK;
}

int styx_residency_hits(const styx_residency *r, int layer, uint64_t *hits) {
    RNEED(r && hits, "null pointer");
    RNEED(layer >= 0 && layer < r->n_layers, "layer %d out of range", layer);
    std::memcpy(hits, r->hits[layer].data(), r->hits[layer].size() * 8);
    return STYX_OK;
}

int styx_residency_maybe_repin(styx_residency *r, const int32_t *ids, uint64_t n_past, uint64_t interval,
                               int max_per_layer, styx_repin_swap *swaps, int cap, int *n_swaps) {
    RNEED(r && ids && n_swaps, "null pointer");
    RNEED(max_per_layer >= 0 && cap >= 0 && (cap == 0 || swaps), "bad max_per_layer / cap");
    RNEED(static_cast<long long>(cap) >= static_cast<long long>(r->n_layers) * max_per_layer,
          "cap %d < n_layers x max_per_layer (%lld): raise cap", cap,
          static_cast<long long>(r->n_layers) * max_per_layer);
    *n_swaps = 0;
    if (interval == 0) return STYX_OK;
    for (int l = 0; l < r->n_layers; l++)
        for (int s = 0; s < r->k; s++) {
            const int e = routed(*r, ids, l, s);
            if (e >= 0) r->hits[l][e]++;
        }
    if (n_past % interval != 0) return STYX_OK;
    int n = 0;
    for (int l = 0; l < r->n_layers; l++) {
        std::vector<uint32_t> &slots = r->slot_experts[l];
        const std::vector<uint64_t> &h = r->hits[l];
        const int n_slots = static_cast<int>(slots.size());
        if (n_slots == 0) continue;
        // residents coldest first (slot order on ties), outsiders hottest
        // first (ascending id on ties)
        std::vector<int> res(n_slots);
        std::iota(res.begin(), res.end(), 0);
        std::stable_sort(res.begin(), res.end(), [&](int a, int b) { return h[slots[a]] < h[slots[b]]; });
        std::vector<uint32_t> out;
        for (int e = 0; e < r->n_expert; e++)
            if (r->remap[l][e] == STYX_SKIP) out.push_back(static_cast<uint32_t>(e));
        std::stable_sort(out.begin(), out.end(), [&](uint32_t a, uint32_t b) { return h[a] > h[b]; });
        const int pairs = std::min({n_slots, static_cast<int>(out.size()), max_per_layer});
        for (int i = 0; i < pairs; i++) {
            const int slot = res[i];
            const uint32_t old = slots[slot], nw = out[i];
            if (h[nw] < 2 * std::max<uint64_t>(h[old], 1)) break;   // hysteresis: ranked lists, no later pair pays
            r->remap[l][old] = STYX_SKIP;
            r->remap[l][nw] = static_cast<uint32_t>(slot);
            slots[slot] = nw;
            swaps[n++] = styx_repin_swap{l, slot, old, nw};
        }
    }
    *n_swaps = n;
    return STYX_OK;
}

int styx_residency_hot_cold(const styx_residency *r, const int32_t *ids, uint32_t *hot, uint32_t *cold) {
    RNEED(r && ids && hot && cold, "null pointer");
    for (int l = 0; l < r->n_layers; l++) {
        uint32_t h = 0;
        for (int s = 0; s < r->k; s++) {
            const int e = routed(*r, ids, l, s);
            if (e >= 0 && r->remap[l][e] != STYX_SKIP) h++;
        }
        hot[l] = h;
        cold[l] = static_cast<uint32_t>(r->k) - h;
    }
    return STYX_OK;
}

int styx_residency_prefetch_plan(const styx_residency *r, const int32_t *ids, uint32_t *pmap, int32_t *pf_ids) {
    RNEED(r && ids && pmap && pf_ids, "null pointer");
    for (int l = 0; l < r->n_layers; l++) {
        uint32_t *pm = pmap + static_cast<size_t>(l) * r->n_expert;
        int32_t *pf = pf_ids + static_cast<size_t>(l) * STYX_IDS_PER_LAYER;
        for (int e = 0; e < r->n_expert; e++) pm[e] = STYX_SKIP;
        int n_pf = 0;
        for (int s = 0; s < r->k; s++) {
            const int e = routed(*r, ids, l, s);
            if (e < 0) continue;                          // SKIP in row 0 (the reference panics)
            if (r->remap[l][e] != STYX_SKIP) continue;    // hot experts read the hot buffer
            if (pm[e] != STYX_SKIP) continue;             // duplicate in this layer
            pm[e] = static_cast<uint32_t>(l * r->k + n_pf);   // global arena slot
            pf[n_pf++] = e;
        }
        for (int s = n_pf; s < r->k; s++) pf[s] = -1;
    }
    return STYX_OK;
}

}  // extern "C"
