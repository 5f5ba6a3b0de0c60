// Host decode runtime: block manager, the scheduler's capacity pass, and the greedy / beam
// bookkeeping of a decode step (declared in vflorence_b200_runtime.h). Host code only.
//
// Decisions follow the reference engine (paths inside the vflorence project):
//   block_manager.py:7-73   free list first-in first-out; ensure_capacity appends a block when
//                           the table is full, or swaps a shared block for a private copy
//                           unless the writer is its last holder; release last block first
//   scheduler.py:35-61      required_new_blocks over the whole step, then ensure_capacity in
//                           running order
//   scheduler.py:63-127     num_cached_tokens += 1 for every row, then greedy append/finish or
//                           the beam split / ranking / early stop / fork / release
//   sequence.py:53-80       fork, num_generated, is_finished, score
#include <algorithm>
#include <cmath>
#include <limits>
#include <new>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "vflorence_b200_runtime.h"

using vfl::fail;

namespace {

struct Hyp {
  int64_t request_id = -1;
  int32_t length = 0;      // decoder tokens, the start token included
  int32_t last_token = 0;
  int32_t num_cached = 0;  // tokens whose K/V are in the pool
  double cum_logprob = 0.0;
  double score = 0.0;      // length-penalised score, set when a beam step creates it
};

struct Finished {
  int32_t slot;
  double score;
};

constexpr int32_t kMaxSlots = 1 << 24;
constexpr int32_t kMaxBlocks = 1 << 30;

}  // namespace

struct vfl_runtime {
  int32_t num_blocks = 0, block_size = 0, num_slots = 0, max_blocks = 0;
  // block manager
  std::vector<int32_t> ref_counts;
  std::vector<int32_t> ring;  // free list: `count` ids from `head`, oldest first
  int32_t head = 0, count = 0;
  std::vector<int32_t> tables;     // [num_slots][max_blocks]
  std::vector<int32_t> table_len;  // [num_slots]
  // hypotheses
  std::vector<Hyp> hyps;
  std::vector<char> slot_used;
  std::vector<int32_t> free_slots;  // stack: the back is handed out next
  std::vector<int32_t> running;
  std::unordered_map<int64_t, std::vector<Finished>> finished;
  // scratch
  std::vector<int32_t> left;     // required_new_blocks: holders not yet counted, -1 = unset
  std::vector<int32_t> touched;
  std::vector<int32_t> rows, group_of, new_running, released;
  std::vector<int64_t> group_rid;
  std::unordered_map<int64_t, int32_t> group_index;

  int32_t* table(int32_t slot) { return tables.data() + (size_t)slot * max_blocks; }
  const int32_t* table(int32_t slot) const { return tables.data() + (size_t)slot * max_blocks; }

  void reset() {
    std::fill(ref_counts.begin(), ref_counts.end(), 0);
    for (int32_t i = 0; i < num_blocks; ++i) ring[i] = i;
    head = 0;
    count = num_blocks;
    std::fill(table_len.begin(), table_len.end(), 0);
    std::fill(slot_used.begin(), slot_used.end(), 0);
    free_slots.resize(num_slots);
    for (int32_t i = 0; i < num_slots; ++i) free_slots[i] = i;
    running.clear();
    finished.clear();
  }

  int take_block(int32_t* block) {
    if (count == 0) return fail(VFL_ERR_CAPACITY, "KV cache is full; increase num_blocks");
    *block = ring[head];
    head = head + 1 == num_blocks ? 0 : head + 1;
    --count;
    ref_counts[*block] = 1;
    return VFL_OK;
  }

  void give_block(int32_t block) {
    int64_t tail = (int64_t)head + count;
    if (tail >= num_blocks) tail -= num_blocks;
    ring[tail] = block;
    ++count;
  }

  int64_t required(const int32_t* slots, const int32_t* cached, int32_t n, bool from_hyps) {
    int64_t needed = 0;
    for (int32_t i = 0; i < n; ++i) {
      const int32_t s = slots[i];
      const int32_t nc = from_hyps ? hyps[s].num_cached : cached[i];
      const int32_t idx = nc / block_size;
      if (idx >= table_len[s]) {
        ++needed;
        continue;
      }
      const int32_t block = table(s)[idx];
      int32_t holders = left[block] >= 0 ? left[block] : ref_counts[block];
      if (holders > 1) {
        ++needed;
        if (left[block] < 0) touched.push_back(block);
        left[block] = holders - 1;
      }
    }
    for (int32_t b : touched) left[b] = -1;
    touched.clear();
    return needed;
  }

  // One slot's next token: the caller has checked the slot and that a block can be taken.
  int ensure(int32_t s, int32_t nc, int32_t* src, int32_t* dst) {
    *src = *dst = -1;
    const int32_t idx = nc / block_size;
    int32_t* t = table(s);
    if (idx > table_len[s])
      return fail(VFL_ERR_INVALID_ARGUMENT, "ensure_capacity: token %d of slot %d skips a block (table has %d)",
                  nc, s, table_len[s]);
    if (idx == table_len[s]) {
      if (table_len[s] == max_blocks)
        return fail(VFL_ERR_INVALID_ARGUMENT, "slot %d: more than %d blocks (max_blocks_per_seq)", s, max_blocks);
      int32_t b;
      int st = take_block(&b);
      if (st) return st;
      t[table_len[s]++] = b;
      return VFL_OK;
    }
    const int32_t block = t[idx];
    if (ref_counts[block] == 1) return VFL_OK;
    int32_t fresh;
    int st = take_block(&fresh);
    if (st) return st;
    --ref_counts[block];
    t[idx] = fresh;
    *src = block;
    *dst = fresh;
    return VFL_OK;
  }

  void fork(int32_t parent, int32_t child) {
    const int32_t n = table_len[parent];
    std::copy(table(parent), table(parent) + n, table(child));
    table_len[child] = n;
    for (int32_t i = 0; i < n; ++i) ++ref_counts[table(child)[i]];
  }

  void deallocate(int32_t s) {
    const int32_t* t = table(s);
    for (int32_t i = table_len[s] - 1; i >= 0; --i)
      if (--ref_counts[t[i]] == 0) give_block(t[i]);
    table_len[s] = 0;
  }

  int32_t pop_slot() {
    const int32_t s = free_slots.back();
    free_slots.pop_back();
    slot_used[s] = 1;
    return s;
  }

  void push_slot(int32_t s) {
    slot_used[s] = 0;
    free_slots.push_back(s);
  }

  // Group (request) index of every running row, in order of first appearance.
  int32_t compute_groups() {
    const size_t n = running.size();
    group_of.resize(n);
    group_rid.clear();
    group_index.clear();
    int64_t prev = std::numeric_limits<int64_t>::min();
    int32_t prev_g = -1;
    for (size_t i = 0; i < n; ++i) {
      const int64_t rid = hyps[running[i]].request_id;
      int32_t g;
      if (rid == prev) {
        g = prev_g;
      } else {
        auto it = group_index.find(rid);
        if (it == group_index.end()) {
          g = (int32_t)group_rid.size();
          group_index.emplace(rid, g);
          group_rid.push_back(rid);
        } else {
          g = it->second;
        }
      }
      group_of[i] = g;
      prev = rid;
      prev_g = g;
    }
    return (int32_t)group_rid.size();
  }
};

namespace {

bool slot_ok(const vfl_runtime* rt, int32_t s) { return s >= 0 && s < rt->num_slots; }

bool is_eos(const vfl_decode_rules* r, int64_t token) {
  for (int32_t i = 0; i < r->num_eos; ++i)
    if (r->eos_ids[i] == token) return true;
  return false;
}

int check_rules(const vfl_decode_rules* r) {
  if (r == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "decode rules are NULL");
  if (r->num_beams < 1 || r->max_tokens < 1)
    return fail(VFL_ERR_INVALID_ARGUMENT, "num_beams and max_tokens must be >= 1");
  if (r->num_eos < 0 || (r->num_eos > 0 && r->eos_ids == nullptr))
    return fail(VFL_ERR_INVALID_ARGUMENT, "eos ids missing");
  return VFL_OK;
}

int check_result(vfl_step_result* out) {
  if (out == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "step result is NULL");
  out->num_born = 0;
  out->num_done = 0;
  return VFL_OK;
}

// sequence.py:76-80: cum_logprob / max(num_generated, 1) ** length_penalty
double length_penalised(double cum, int32_t num_generated, double length_penalty) {
  return cum / std::pow((double)std::max(num_generated, 1), length_penalty);
}

}  // namespace

extern "C" {

int vfl_rt_create(int32_t num_blocks, int32_t block_size, int32_t num_slots, int32_t max_blocks_per_seq,
                  vfl_runtime** out) {
  if (out == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  if (num_blocks <= 0 || num_blocks > kMaxBlocks || block_size <= 0 || num_slots <= 0 || num_slots > kMaxSlots ||
      max_blocks_per_seq <= 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "runtime sizes out of range (blocks %d, block_size %d, slots %d, "
                "max_blocks_per_seq %d)", num_blocks, block_size, num_slots, max_blocks_per_seq);
  if ((int64_t)num_slots * max_blocks_per_seq > ((int64_t)1 << 31))
    return fail(VFL_ERR_INVALID_ARGUMENT, "num_slots * max_blocks_per_seq too large");
  vfl_runtime* rt = new (std::nothrow) vfl_runtime();
  if (rt == nullptr) return fail(VFL_ERR_CAPACITY, "out of host memory");
  try {
    rt->num_blocks = num_blocks;
    rt->block_size = block_size;
    rt->num_slots = num_slots;
    rt->max_blocks = max_blocks_per_seq;
    rt->ref_counts.assign(num_blocks, 0);
    rt->ring.assign(num_blocks, 0);
    rt->left.assign(num_blocks, -1);
    rt->tables.assign((size_t)num_slots * max_blocks_per_seq, 0);
    rt->table_len.assign(num_slots, 0);
    rt->hyps.assign(num_slots, Hyp());
    rt->slot_used.assign(num_slots, 0);
    rt->reset();
  } catch (const std::bad_alloc&) {
    delete rt;
    return fail(VFL_ERR_CAPACITY, "out of host memory");
  }
  *out = rt;
  return VFL_OK;
}

void vfl_rt_destroy(vfl_runtime* rt) { delete rt; }

int vfl_rt_reset(vfl_runtime* rt) {
  if (rt == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "runtime is NULL");
  rt->reset();
  return VFL_OK;
}

// ----------------------------------------------------------------------------- block manager
int vfl_rt_slot_acquire(vfl_runtime* rt, int32_t* slot) {
  if (rt == nullptr || slot == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "NULL argument");
  if (rt->free_slots.empty()) return fail(VFL_ERR_CAPACITY, "no free hypothesis slot (num_slots %d)", rt->num_slots);
  *slot = rt->pop_slot();
  rt->hyps[*slot] = Hyp();
  return VFL_OK;
}

int vfl_rt_slot_release(vfl_runtime* rt, int32_t slot) {
  if (rt == nullptr || !slot_ok(rt, slot) || !rt->slot_used[slot])
    return fail(VFL_ERR_INVALID_ARGUMENT, "slot %d is not in use", slot);
  if (rt->table_len[slot] != 0) return fail(VFL_ERR_INVALID_ARGUMENT, "slot %d still holds blocks", slot);
  rt->push_slot(slot);
  return VFL_OK;
}

int vfl_rt_num_free_blocks(const vfl_runtime* rt, int32_t* out) {
  if (rt == nullptr || out == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "NULL argument");
  *out = rt->count;
  return VFL_OK;
}

int vfl_rt_free_block_ids(const vfl_runtime* rt, int32_t* out, int32_t cap, int32_t* n) {
  if (rt == nullptr || n == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "NULL argument");
  *n = rt->count;
  if (cap < rt->count || (rt->count > 0 && out == nullptr))
    return fail(VFL_ERR_INVALID_ARGUMENT, "free_block_ids: capacity %d < %d", cap, rt->count);
  int32_t h = rt->head;
  for (int32_t i = 0; i < rt->count; ++i) {
    out[i] = rt->ring[h];
    h = h + 1 == rt->num_blocks ? 0 : h + 1;
  }
  return VFL_OK;
}

int vfl_rt_ref_count(const vfl_runtime* rt, int32_t block, int32_t* out) {
  if (rt == nullptr || out == nullptr || block < 0 || block >= rt->num_blocks)
    return fail(VFL_ERR_INVALID_ARGUMENT, "ref_count: bad block %d", block);
  *out = rt->ref_counts[block];
  return VFL_OK;
}

int vfl_rt_block_table(const vfl_runtime* rt, int32_t slot, int32_t* out, int32_t cap, int32_t* n) {
  if (rt == nullptr || n == nullptr || !slot_ok(rt, slot))
    return fail(VFL_ERR_INVALID_ARGUMENT, "block_table: bad slot %d", slot);
  *n = rt->table_len[slot];
  if (cap < *n || (*n > 0 && out == nullptr))
    return fail(VFL_ERR_INVALID_ARGUMENT, "block_table: capacity %d < %d", cap, *n);
  std::copy(rt->table(slot), rt->table(slot) + *n, out);
  return VFL_OK;
}

int vfl_rt_required_new_blocks(const vfl_runtime* rt, const int32_t* slots, const int32_t* num_cached, int32_t n,
                               int64_t* out) {
  if (rt == nullptr || out == nullptr || n < 0 || (n > 0 && (slots == nullptr || num_cached == nullptr)))
    return fail(VFL_ERR_INVALID_ARGUMENT, "required_new_blocks: NULL argument");
  for (int32_t i = 0; i < n; ++i)
    if (!slot_ok(rt, slots[i]) || num_cached[i] < 0)
      return fail(VFL_ERR_INVALID_ARGUMENT, "required_new_blocks: bad slot %d / count %d", slots[i], num_cached[i]);
  *out = const_cast<vfl_runtime*>(rt)->required(slots, num_cached, n, false);
  return VFL_OK;
}

int vfl_rt_ensure_capacity(vfl_runtime* rt, int32_t slot, int32_t num_cached, int32_t* src, int32_t* dst) {
  if (rt == nullptr || src == nullptr || dst == nullptr || !slot_ok(rt, slot) || num_cached < 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "ensure_capacity: bad argument (slot %d, count %d)", slot, num_cached);
  return rt->ensure(slot, num_cached, src, dst);
}

int vfl_rt_fork(vfl_runtime* rt, int32_t parent, int32_t child) {
  if (rt == nullptr || !slot_ok(rt, parent) || !slot_ok(rt, child) || parent == child)
    return fail(VFL_ERR_INVALID_ARGUMENT, "fork: bad slots %d -> %d", parent, child);
  if (rt->table_len[child] != 0) return fail(VFL_ERR_INVALID_ARGUMENT, "fork: child slot %d holds blocks", child);
  rt->fork(parent, child);
  return VFL_OK;
}

int vfl_rt_deallocate(vfl_runtime* rt, int32_t slot) {
  if (rt == nullptr || !slot_ok(rt, slot)) return fail(VFL_ERR_INVALID_ARGUMENT, "deallocate: bad slot %d", slot);
  rt->deallocate(slot);
  return VFL_OK;
}

// ------------------------------------------------------------------------ decode hypotheses
int vfl_rt_admit(vfl_runtime* rt, int64_t request_id, int32_t start_token, int32_t* slot) {
  if (rt == nullptr || slot == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "admit: NULL argument");
  if (rt->free_slots.empty()) return fail(VFL_ERR_CAPACITY, "no free hypothesis slot (num_slots %d)", rt->num_slots);
  const int32_t s = rt->pop_slot();
  Hyp& h = rt->hyps[s];
  h = Hyp();
  h.request_id = request_id;
  h.length = 1;
  h.last_token = start_token;
  rt->table_len[s] = 0;
  rt->running.push_back(s);
  *slot = s;
  return VFL_OK;
}

int vfl_rt_num_running(const vfl_runtime* rt, int32_t* out) {
  if (rt == nullptr || out == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "NULL argument");
  *out = (int32_t)rt->running.size();
  return VFL_OK;
}

int vfl_rt_prepare_step(vfl_runtime* rt, int32_t* pairs, int32_t cap, int32_t* num_pairs) {
  if (rt == nullptr || num_pairs == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "prepare_step: NULL argument");
  *num_pairs = 0;
  const int32_t n = (int32_t)rt->running.size();
  if (n > 0 && (pairs == nullptr || cap < n))
    return fail(VFL_ERR_INVALID_ARGUMENT, "prepare_step: pair capacity %d < running %d", cap, n);
  for (int32_t s : rt->running) {
    const int32_t idx = rt->hyps[s].num_cached / rt->block_size;
    if (idx > rt->table_len[s] || (idx == rt->table_len[s] && idx == rt->max_blocks))
      return fail(VFL_ERR_INVALID_ARGUMENT, "prepare_step: slot %d at token %d does not fit its table", s,
                  rt->hyps[s].num_cached);
  }
  if (rt->required(rt->running.data(), nullptr, n, true) > rt->count)
    return fail(VFL_ERR_CAPACITY, "KV cache is full; increase num_blocks");
  for (int32_t s : rt->running) {
    int32_t src, dst;
    int st = rt->ensure(s, rt->hyps[s].num_cached, &src, &dst);
    if (st) return st;  // unreachable: the capacity and the tables were checked above
    if (src >= 0) {
      pairs[2 * *num_pairs] = src;
      pairs[2 * *num_pairs + 1] = dst;
      ++*num_pairs;
    }
  }
  return VFL_OK;
}

int vfl_rt_pack_step(const vfl_runtime* crt, int32_t cap, int32_t* tables, int64_t table_stride, int32_t width,
                     int32_t* table_lens, int32_t* positions, int32_t* tokens, int32_t* slots, int32_t* lengths,
                     int64_t* request_ids, int32_t* groups, int32_t* ranks, float* cum_logprobs,
                     int32_t* num_groups, int32_t* max_rank) {
  if (crt == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "pack_step: runtime is NULL");
  vfl_runtime* rt = const_cast<vfl_runtime*>(crt);
  const int32_t n = (int32_t)rt->running.size();
  if (cap < n) return fail(VFL_ERR_INVALID_ARGUMENT, "pack_step: capacity %d < running %d", cap, n);
  if (tables != nullptr) {
    if (width < 0 || table_stride < width)
      return fail(VFL_ERR_INVALID_ARGUMENT, "pack_step: table width %d / stride %lld", width, (long long)table_stride);
    for (int32_t i = 0; i < n; ++i)
      if (rt->table_len[rt->running[i]] > width)
        return fail(VFL_ERR_INVALID_ARGUMENT, "pack_step: table of %d blocks wider than %d",
                    rt->table_len[rt->running[i]], width);
  }
  const int32_t ng = rt->compute_groups();
  std::vector<int32_t> seen(ng, 0);
  int32_t mr = 0;
  for (int32_t i = 0; i < n; ++i) {
    const int32_t s = rt->running[i];
    const Hyp& h = rt->hyps[s];
    if (tables != nullptr) {
      int32_t* row = tables + (int64_t)i * table_stride;
      const int32_t len = rt->table_len[s];
      std::copy(rt->table(s), rt->table(s) + len, row);
      std::fill(row + len, row + width, 0);
    }
    if (table_lens) table_lens[i] = rt->table_len[s];
    if (positions) positions[i] = h.num_cached;
    if (tokens) tokens[i] = h.last_token;
    if (slots) slots[i] = s;
    if (lengths) lengths[i] = h.length;
    if (request_ids) request_ids[i] = h.request_id;
    const int32_t g = rt->group_of[i];
    if (groups) groups[i] = g;
    const int32_t r = seen[g]++;
    if (ranks) ranks[i] = r;
    mr = std::max(mr, r + 1);
    if (cum_logprobs) cum_logprobs[i] = (float)h.cum_logprob;
  }
  if (num_groups) *num_groups = ng;
  if (max_rank) *max_rank = mr;
  return VFL_OK;
}

int vfl_rt_advance_greedy(vfl_runtime* rt, const vfl_decode_rules* rules, const int64_t* picks, int32_t n,
                          vfl_step_result* out) {
  if (rt == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "advance_greedy: runtime is NULL");
  int st = check_rules(rules);
  if (st) return st;
  if ((st = check_result(out))) return st;
  if (n != (int32_t)rt->running.size() || (n > 0 && picks == nullptr))
    return fail(VFL_ERR_INVALID_ARGUMENT, "advance_greedy: %d picks for %zu running rows", n, rt->running.size());
  int32_t done = 0;
  for (int32_t i = 0; i < n; ++i) {
    const Hyp& h = rt->hyps[rt->running[i]];
    done += (is_eos(rules, picks[i]) || h.length >= rules->max_tokens) ? 1 : 0;
  }
  if (done > out->done_cap) return fail(VFL_ERR_INVALID_ARGUMENT, "advance_greedy: done capacity %d < %d",
                                        out->done_cap, done);
  rt->new_running.clear();
  for (int32_t i = 0; i < n; ++i) {
    const int32_t s = rt->running[i];
    Hyp& h = rt->hyps[s];
    ++h.num_cached;
    h.last_token = (int32_t)picks[i];
    ++h.length;
    if (is_eos(rules, picks[i]) || h.length - 1 >= rules->max_tokens) {
      out->done_request[out->num_done] = h.request_id;
      out->done_slot[out->num_done] = s;
      out->done_length[out->num_done] = h.length;
      ++out->num_done;
    } else {
      rt->new_running.push_back(s);
    }
  }
  for (int32_t i = 0; i < out->num_done; ++i) {
    rt->deallocate(out->done_slot[i]);
    rt->push_slot(out->done_slot[i]);
  }
  rt->running.swap(rt->new_running);
  return VFL_OK;
}

int vfl_rt_advance_beam(vfl_runtime* rt, const vfl_decode_rules* rules, const int32_t* cand_row,
                        const int32_t* cand_token, const float* cand_score, int32_t num_groups, int32_t per_group,
                        vfl_step_result* out) {
  if (rt == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "advance_beam: runtime is NULL");
  int st = check_rules(rules);
  if (st) return st;
  if ((st = check_result(out))) return st;
  const int32_t n = (int32_t)rt->running.size();
  const int32_t ng = rt->compute_groups();
  if (num_groups != ng || per_group < 1 || (ng > 0 && (!cand_row || !cand_token || !cand_score)))
    return fail(VFL_ERR_INVALID_ARGUMENT, "advance_beam: %d groups x %d candidates for %d requests", num_groups,
                per_group, ng);
  const int64_t total = (int64_t)ng * per_group;
  for (int32_t g = 0; g < ng; ++g) {
    if (cand_row[(int64_t)g * per_group] < 0)
      return fail(VFL_ERR_INVALID_ARGUMENT, "advance_beam: request group %d has no candidate", g);
    for (int32_t j = 0; j < per_group; ++j) {
      const int32_t row = cand_row[(int64_t)g * per_group + j];
      if (row >= n || (row >= 0 && rt->group_of[row] != g))
        return fail(VFL_ERR_INVALID_ARGUMENT, "advance_beam: candidate row %d is not a row of request group %d",
                    row, g);
    }
  }
  if ((int64_t)rt->free_slots.size() < total)
    return fail(VFL_ERR_CAPACITY, "advance_beam: %zu free hypothesis slots for up to %lld children",
                rt->free_slots.size(), (long long)total);
  if (out->born_cap < total || out->done_cap < ng)
    return fail(VFL_ERR_INVALID_ARGUMENT, "advance_beam: result capacity (born %d, done %d) below %lld / %d",
                out->born_cap, out->done_cap, (long long)total, ng);

  const int32_t nb = rules->num_beams;
  rt->rows.assign(rt->running.begin(), rt->running.end());
  for (int32_t s : rt->rows) ++rt->hyps[s].num_cached;
  rt->new_running.clear();
  rt->released.clear();
  std::vector<std::pair<int32_t, int32_t>> running_children;
  for (int32_t g = 0; g < ng; ++g) {
    const int64_t rid = rt->group_rid[g];
    std::vector<Finished>& fin = rt->finished[rid];
    running_children.clear();
    int32_t rank = 0;
    for (int32_t j = 0; j < per_group; ++j) {
      const int64_t c = (int64_t)g * per_group + j;
      const int32_t row = cand_row[c];
      if (row < 0) continue;
      if (rank >= nb && (int32_t)running_children.size() >= nb) break;
      const int32_t r = rank++;
      const int32_t parent = rt->rows[row];
      const Hyp& p = rt->hyps[parent];
      const int32_t token = cand_token[c];
      const bool done = is_eos(rules, token) || p.length >= rules->max_tokens;  // child's generated count
      if (done && r >= nb) continue;
      if (!done && (int32_t)running_children.size() >= nb) continue;
      const int32_t child = rt->pop_slot();
      Hyp& h = rt->hyps[child];
      h.request_id = rid;
      h.length = p.length + 1;
      h.last_token = token;
      h.num_cached = p.num_cached;
      h.cum_logprob = (double)cand_score[c];
      h.score = length_penalised(h.cum_logprob, h.length - 1, rules->length_penalty);
      rt->table_len[child] = 0;
      out->born_parent[out->num_born] = parent;
      out->born_child[out->num_born] = child;
      out->born_pos[out->num_born] = p.length;
      out->born_token[out->num_born] = token;
      ++out->num_born;
      if (done)
        fin.push_back({child, h.score});
      else
        running_children.emplace_back(parent, child);
    }
    std::stable_sort(fin.begin(), fin.end(),
                     [](const Finished& a, const Finished& b) { return a.score > b.score; });
    for (size_t k = nb; k < fin.size(); ++k) rt->released.push_back(fin[k].slot);
    if ((int32_t)fin.size() > nb) fin.resize(nb);
    // the best running score: the first child's, replaced by any larger one (Python's max)
    double best_running = -std::numeric_limits<double>::infinity();
    for (size_t k = 0; k < running_children.size(); ++k) {
      const double sc = rt->hyps[running_children[k].second].score;
      if (k == 0 || sc > best_running) best_running = sc;
    }
    const bool stop = (int32_t)fin.size() >= nb && (rules->early_stopping || fin.back().score >= best_running);
    if (running_children.empty() || stop) {
      const int32_t best = fin.front().slot;  // non-empty: the first candidate is kept either way
      out->done_request[out->num_done] = rid;
      out->done_slot[out->num_done] = best;
      out->done_length[out->num_done] = rt->hyps[best].length;
      ++out->num_done;
      for (const Finished& f : fin) rt->released.push_back(f.slot);
      for (auto& pc : running_children) rt->released.push_back(pc.second);
      rt->finished.erase(rid);
    } else {
      for (auto& pc : running_children) {
        rt->fork(pc.first, pc.second);
        rt->new_running.push_back(pc.second);
      }
    }
  }
  // every parent leaves: blocks released in row order, then the parents' and the released
  // hypotheses' slots return to the free stack
  for (int32_t s : rt->rows) {
    rt->deallocate(s);
    rt->push_slot(s);
  }
  for (int32_t s : rt->released) rt->push_slot(s);
  rt->running.swap(rt->new_running);
  return VFL_OK;
}

}  // extern "C"
