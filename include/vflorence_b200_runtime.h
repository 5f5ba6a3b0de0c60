/*
 * vflorence_b200 host decode runtime: the per-step bookkeeping of the paged decode loop in
 * native code, on the host. It owns no device memory; what it decides (block tables, slots,
 * copy-on-write pairs, which hypotheses live on) is what the device ops of
 * vflorence_b200.h consume.
 *
 * It replaces these pieces of the reference engine (paths inside the vflorence project):
 *
 *   BlockManager                 vflorence/engine/block_manager.py:7-73
 *       free block ids handed out first-in first-out, reference counts, copy-on-write of a
 *       shared block for every holder but the last, release of a table last block first
 *   Scheduler.schedule (part)    vflorence/engine/scheduler.py:35-61
 *       capacity check for the whole step, then ensure_capacity in running order
 *   Scheduler.postprocess        vflorence/engine/scheduler.py:63-127
 *       greedy append/finish, and the beam split into finished and running hypotheses, the
 *       length-penalised ranking of finished ones, the early-stop rule, forks of the kept
 *       children and the release of every parent
 *   Sequence bookkeeping         vflorence/engine/sequence.py:50-80
 *       append/fork, num_generated, is_finished, score
 *
 * A hypothesis (the reference's Sequence) is addressed by its slot: an integer in
 * [0, num_slots) that the caller also uses as the row of its device token buffer. Slots are
 * handed out last-freed first. Token ids themselves live on the device; the runtime keeps a
 * hypothesis's length, last token, cached-token count, cumulative log-prob and block table.
 *
 * Every function returns a vfl_status (vflorence_b200.h); the message of a failure is
 * available from vfl_last_error_message(). A runtime object is not thread-safe: one caller
 * thread at a time.
 */
#ifndef VFLORENCE_B200_RUNTIME_H_
#define VFLORENCE_B200_RUNTIME_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct vfl_runtime vfl_runtime;

/* Creates a runtime over a pool of `num_blocks` blocks of `block_size` tokens, `num_slots`
 * hypothesis slots, and block tables of at most `max_blocks_per_seq` entries.
 * Replaces BlockManager.__init__ (block_manager.py:7-16). */
int vfl_rt_create(int32_t num_blocks, int32_t block_size, int32_t num_slots,
                  int32_t max_blocks_per_seq, vfl_runtime** out);
void vfl_rt_destroy(vfl_runtime* rt);
/* Frees every block, slot and hypothesis (block_manager.py:12-16 plus the scheduler's reset,
 * scheduler.py:21-26). */
int vfl_rt_reset(vfl_runtime* rt);

/* ------------------------------------------------------------------------ block manager */
/* The BlockManager interface on single slots, for callers that keep their own sequences
 * (block_manager.py:18-73). `vfl_rt_slot_acquire` / `vfl_rt_slot_release` hand out slots
 * without creating a decoding hypothesis. */
int vfl_rt_slot_acquire(vfl_runtime* rt, int32_t* slot);
int vfl_rt_slot_release(vfl_runtime* rt, int32_t slot);
int vfl_rt_num_free_blocks(const vfl_runtime* rt, int32_t* out);
/* The free list in hand-out order (oldest first); `*n` receives its length. */
int vfl_rt_free_block_ids(const vfl_runtime* rt, int32_t* out, int32_t cap, int32_t* n);
int vfl_rt_ref_count(const vfl_runtime* rt, int32_t block, int32_t* out);
int vfl_rt_block_table(const vfl_runtime* rt, int32_t slot, int32_t* out, int32_t cap, int32_t* n);
/* block_manager.py:28-42: blocks that appending one token to each listed slot (with the
 * given cached-token counts) would take. */
int vfl_rt_required_new_blocks(const vfl_runtime* rt, const int32_t* slots,
                               const int32_t* num_cached, int32_t n, int64_t* out);
/* block_manager.py:44-59: makes the block of token `num_cached` writable. `*src`/`*dst`
 * receive the copy-on-write pair, or -1/-1. VFL_ERR_CAPACITY when no block is free. */
int vfl_rt_ensure_capacity(vfl_runtime* rt, int32_t slot, int32_t num_cached, int32_t* src,
                           int32_t* dst);
/* block_manager.py:61-65: `child` shares every block of `parent`. */
int vfl_rt_fork(vfl_runtime* rt, int32_t parent, int32_t child);
/* block_manager.py:67-73: drops the slot's references, last block first. */
int vfl_rt_deallocate(vfl_runtime* rt, int32_t slot);

/* ---------------------------------------------------------------------- decode hypotheses */
/* Decoding rules the bookkeeping needs (the rest of SamplingParams acts on device logits). */
typedef struct vfl_decode_rules {
  int32_t num_beams;
  int32_t max_tokens;
  double length_penalty;
  int32_t early_stopping;
  int32_t num_eos;
  const int32_t* eos_ids; /* num_eos entries */
} vfl_decode_rules;

/* Admits a request as one running hypothesis holding the decoder start token (length 1),
 * appended to the running list (scheduler.py:42-48). `*slot` receives its slot. */
int vfl_rt_admit(vfl_runtime* rt, int64_t request_id, int32_t start_token, int32_t* slot);
int vfl_rt_num_running(const vfl_runtime* rt, int32_t* out);

/* scheduler.py:50-61: room for every running hypothesis's next token, in running order.
 * All or nothing: VFL_ERR_CAPACITY (nothing changed) when the step needs more blocks than are
 * free. Copy-on-write pairs go to `pairs` ([cap][2] src, dst); `*num_pairs` receives their
 * count (at most the number of running hypotheses). */
int vfl_rt_prepare_step(vfl_runtime* rt, int32_t* pairs, int32_t cap, int32_t* num_pairs);

/* The running hypotheses' step inputs, row i = i-th running hypothesis. Any output may be
 * NULL. tables: [n, width] rows at `table_stride` int32, zero-padded (model_runner.py:302-304);
 * table_lens: entries per table; positions: cached-token counts (the new token's position);
 * tokens: last tokens; slots; lengths: decoder tokens incl. the start token; request_ids;
 * groups: index of the row's request in order of first appearance; ranks: index of the row
 * among its request's rows; cum_logprobs. `*num_groups` receives the number of requests and
 * `*max_rank` the largest rank + 1. VFL_ERR_INVALID_ARGUMENT when a table is wider than
 * `width` or `cap` < the running count. */
int vfl_rt_pack_step(const vfl_runtime* rt, int32_t cap, int32_t* tables, int64_t table_stride,
                     int32_t width, int32_t* table_lens, int32_t* positions, int32_t* tokens,
                     int32_t* slots, int32_t* lengths, int64_t* request_ids, int32_t* groups,
                     int32_t* ranks, float* cum_logprobs, int32_t* num_groups, int32_t* max_rank);

/* What a step decided. Caller-owned arrays with the stated capacities.
 *   born_*:  new hypotheses whose device token row must be written: row `born_child` = row
 *            `born_parent` with `born_token` at index `born_pos` (greedy steps append in place:
 *            parent == child).
 *   done_*:  requests finished this step: request id, the emitted hypothesis's slot and
 *            length. Emitted slots are already free again; their device rows keep their
 *            tokens until the next admit or step writes them. */
typedef struct vfl_step_result {
  int32_t* born_parent;
  int32_t* born_child;
  int32_t* born_pos;
  int32_t* born_token;
  int32_t born_cap;
  int32_t num_born;
  int64_t* done_request;
  int32_t* done_slot;
  int32_t* done_length;
  int32_t done_cap;
  int32_t num_done;
} vfl_step_result;

/* scheduler.py:63-81: every running hypothesis takes `picks[i]` (row i of the last pack);
 * finished ones leave the running list, their blocks freed in running order. */
int vfl_rt_advance_greedy(vfl_runtime* rt, const vfl_decode_rules* rules, const int64_t* picks,
                          int32_t n, vfl_step_result* out);

/* scheduler.py:63-70 and :83-127 with the candidates of model_runner.py:383-410: for each of
 * `num_groups` requests (in the pack's group order), up to `per_group` candidates sorted by
 * score: `cand_row` (row of the last pack, < 0 = none), `cand_token`, `cand_score` (the
 * child's cumulative log-prob). */
int vfl_rt_advance_beam(vfl_runtime* rt, const vfl_decode_rules* rules, const int32_t* cand_row,
                        const int32_t* cand_token, const float* cand_score, int32_t num_groups,
                        int32_t per_group, vfl_step_result* out);

#ifdef __cplusplus
}
#endif

#endif /* VFLORENCE_B200_RUNTIME_H_ */
