/*
 * styx_residency.h -- host-side expert residency planning for the MoE block,
 * part of libstyx_moe.so.
 *
 * These are the placement decisions MoeModel makes in
 * crates/model/src/moe.rs: the auto expert budget, popularity pinning
 * (MOE_EXPERT_HIST), the per-layer hot tables the router remaps through,
 * online repinning (MOE_REPIN_INTERVAL / MOE_REPIN_MAX), the HUD hot/cold
 * counts and the prefetch plan (pmap + predicted ids).  The functions work on
 * host arrays only and touch no device: the caller applies a decision with
 * the styx_moe.h entry points, as MoeModel applies its own with copy_region
 * and upload (a repin swap = three styx_copy calls, full slab -> hot slot,
 * plus an upload of the layer's remap table).
 *
 * `ids` arguments are the ids buffer read back after a token: n_layers
 * blocks of STYX_IDS_PER_LAYER int32, row 0 (the first k entries of each
 * block) holding the routed expert ids (MoeModel::last_expert_ids,
 * moe.rs:2386-2400).  An id outside [0, n_expert) (SKIP) is ignored where the
 * reference would index out of bounds.
 *
 * Order of equal counts.  The reference ranks with Rust's unstable sorts,
 * which leave the order of equal hit counts unspecified; here equal counts
 * keep a defined order: input order for pinning, slot order for residents
 * and ascending expert id for outsiders when repinning.
 */
#ifndef STYX_RESIDENCY_H
#define STYX_RESIDENCY_H

#include <stddef.h>
#include <stdint.h>

#include "styx_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Expert VRAM budget of MoeModel::load (moe.rs:741-753): all_vram ->
 * UINT64_MAX (MOE_EXPERTS_VRAM=1); else explicit_bytes when has_explicit
 * (MOE_EXPERTS_VRAM_MB, 0 allowed); else the auto budget
 * device_vram - (headroom + pinned + kv_max + arena), saturating at 0. */
uint64_t styx_expert_budget(uint64_t device_vram, uint64_t headroom_bytes,
                            uint64_t pinned_bytes, uint64_t kv_max_bytes,
                            uint64_t arena_bytes, int has_explicit,
                            uint64_t explicit_bytes, int all_vram);

/* Arena reservation (moe.rs:727-740): n_layers * k * (max gate slab + max
 * up slab + max down slab over the layers). */
uint64_t styx_arena_bytes(int n_layers, int k, const uint64_t max_slab[3]);

typedef struct styx_residency styx_residency;

/* cost_per_expert: bytes one (layer, expert) pin takes from the budget, the
 * sum of layer 0's three slabs (moe.rs:794-800). */
int styx_residency_create(int n_layers, int n_expert, int k,
                          uint64_t cost_per_expert, styx_residency **out);
void styx_residency_destroy(styx_residency *r);

/* Popularity pinning (moe.rs:776-813) from n (layer, expert, hits) entries:
 * entries ranked by hits, hottest first, each pinned while the remaining
 * budget covers cost_per_expert (the first one that does not fit ends it).
 * Each layer's hot slots hold its pinned experts in ascending id order
 * (hot_order, moe.rs:825-835).  Replaces any earlier pinning and resets the
 * repin hit counters.  Entries with a layer or expert out of range are
 * rejected (STYX_EINVAL). */
int styx_residency_pin(styx_residency *r, const int32_t *layer,
                       const int32_t *expert, const uint64_t *hits, int n,
                       uint64_t budget, int *n_pinned);
/* The same from MOE_EXPERT_HIST text: a header line, then "layer,expert,hits"
 * lines; lines that do not parse are skipped, as the reference's
 * filter_map does (moe.rs:781-792). */
int styx_residency_pin_csv(styx_residency *r, const char *text, size_t len,
                           uint64_t budget, int *n_pinned);

/* One layer's tables (moe.rs:984-995): remap u32[n_expert] (hot slot or
 * STYX_SKIP, the table the kernels read), slot_experts u32[n_slots] (the
 * expert resident in each hot slot; may be NULL), n_slots. */
int styx_residency_layer(const styx_residency *r, int layer, uint32_t *remap,
                         uint32_t *slot_experts, int *n_slots);
/* Per-expert hit counters of one layer, u64[n_expert]. */
int styx_residency_hits(const styx_residency *r, int layer, uint64_t *hits);

/* One slab swap decided by a repin: hot slot `slot` of `layer` now holds
 * new_expert (copy each of the three tensors' slab new_expert of the full
 * tensor into hot slot `slot`); old_expert went back to the full tensor. */
typedef struct styx_repin_swap {
    int32_t layer;
    int32_t slot;
    uint32_t old_expert;
    uint32_t new_expert;
} styx_repin_swap;

/* MoeModel::maybe_repin (moe.rs:1450-1505), called before a token with
 * n_past tokens already forwarded and the previous token's ids: nothing when
 * interval == 0; else the previous token's ids are counted, and when
 * n_past % interval == 0 every layer swaps its coldest residents for its
 * hottest outsiders, at most max_per_layer swaps, stopping at the first pair
 * where the outsider has fewer than 2 x max(resident hits, 1) hits.  The
 * swaps are applied to the tables and written to `swaps`; cap must be at
 * least n_layers * max_per_layer (checked first: STYX_EINVAL, nothing
 * changed). */
int styx_residency_maybe_repin(styx_residency *r, const int32_t *ids,
                               uint64_t n_past, uint64_t interval,
                               int max_per_layer, styx_repin_swap *swaps,
                               int cap, int *n_swaps);

/* MoeModel::last_hot_cold (moe.rs:1512-1521): per layer, how many of the k
 * routed ids are pinned (hot) and how many are not (cold). */
int styx_residency_hot_cold(const styx_residency *r, const int32_t *ids,
                            uint32_t *hot, uint32_t *cold);

/* MoeModel::prepare_prefetch's plan (moe.rs:2169-2213): predict the next
 * token's experts as this token's; per layer, every routed expert that is
 * not hot gets the next arena slot layer*k + n (duplicates once).
 * pmap u32[n_layers * n_expert] (arena slot or STYX_SKIP), pf_ids
 * int32[n_layers * STYX_IDS_PER_LAYER] (rows of predicted ids, padded with
 * -1 = SKIP to k; entries past k are left untouched). */
int styx_residency_prefetch_plan(const styx_residency *r, const int32_t *ids,
                                 uint32_t *pmap, int32_t *pf_ids);

#ifdef __cplusplus
}
#endif
#endif
