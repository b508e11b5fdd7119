// kvpool.cpp -- host-side KV page pool (refcounted block ids) and the radix
// prefix cache over pages.
//
// The reference keeps one contiguous KV buffer per request
// (crates/higgs-models/src/cache.rs:130-312) and its PrefixCache stores whole
// cloned caches in a compressed radix trie over token ids
// (crates/higgs-engine/src/prompt_cache.rs:41-311).  Here a cache entry holds
// page ids instead: a hit retains the shared pages (no copy), and because only
// full 16-token pages are ever stored, a page in the cache is immutable --
// appending to a sequence always writes a page that sequence owns alone.
// Trie semantics follow prompt_cache.rs: MIN_PREFIX_LEN = 16 (line 8), the
// deepest match at depth >= 16 wins (find_deepest_match 68-98; here extended to
// prefixes that end inside an edge, served from a cached descendant's pages), edges
// split on partial matches (insert 224-270), least-recently-used eviction
// beyond max entries (evict_lru 280-287) followed by pruning / compression
// (prune 139-158).  Access time is a logical clock, not wall time.
#include <stdint.h>

#include <algorithm>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/higgs_cuda.h"

namespace higgs {
int fail(int code, const std::string& msg);
}
using higgs::fail;

struct higgs_block_pool {
  std::vector<int32_t> refcount;
  std::vector<int32_t> free_list;  // LIFO
};

namespace {

constexpr int kMinPrefix = 16;
constexpr int kPage = HIGGS_PAGE_SIZE;

struct Node {
  std::vector<int32_t> edge;
  bool cached = false;
  std::vector<int32_t> pages;  // pages of the prefix ending here (depth / 16 of them)
  uint64_t last_access = 0;
  std::map<int32_t, std::unique_ptr<Node>> children;
};

}  // namespace

struct higgs_prefix_cache {
  higgs_block_pool* pool = nullptr;
  Node root;
  int num_cached = 0;
  int max_cached = 0;
  uint64_t clock = 0;
};

namespace {

void pool_release(higgs_block_pool* p, const std::vector<int32_t>& pages) {
  for (int32_t pg : pages) {
    if (pg < 0 || pg >= (int32_t)p->refcount.size() || p->refcount[pg] <= 0) continue;
    if (--p->refcount[pg] == 0) p->free_list.push_back(pg);
  }
}

void pool_retain(higgs_block_pool* p, const std::vector<int32_t>& pages) {
  for (int32_t pg : pages) p->refcount[pg]++;
}

// any cached node in n's subtree (its pages begin with the pages of every prefix of it)
const Node* any_cached(const Node& n) {
  if (n.cached) return &n;
  for (const auto& kv : n.children)
    if (const Node* c = any_cached(*kv.second)) return c;
  return nullptr;
}

// Longest reusable prefix of the query, in whole pages.  The reference matches only
// cached nodes whose whole token sequence prefixes the query (find_deepest_match);
// with immutable pages any matched prefix -- ending inside an edge or at an internal
// node -- can also be served from the leading pages of a cached descendant.  Returns
// the node whose pages to use; *best_depth = tokens matched (a multiple of 16).
const Node* find_deepest(const Node& n, const int32_t* tok, int len, int depth, int* best_depth) {
  const Node* best = nullptr;
  int bd = 0;
  if (depth >= kMinPrefix) {
    const int m = depth / kPage * kPage;
    if (n.cached && m == depth) {
      best = &n;
      bd = depth;
    } else if (m >= kMinPrefix) {
      best = any_cached(n);
      bd = best ? m : 0;
    }
  }
  if (depth < len) {
    auto it = n.children.find(tok[depth]);
    if (it != n.children.end()) {
      const Node& c = *it->second;
      int common = 0;
      while (common < (int)c.edge.size() && depth + common < len &&
             c.edge[common] == tok[depth + common])
        ++common;
      if (common == (int)c.edge.size()) {
        int d = 0;
        const Node* deeper = find_deepest(c, tok, len, depth + common, &d);
        if (deeper && d > bd) {
          best = deeper;
          bd = d;
        }
      } else {
        const int m = (depth + common) / kPage * kPage;
        if (m >= kMinPrefix && m > bd) {
          if (const Node* src = any_cached(c)) {
            best = src;
            bd = m;
          }
        }
      }
    }
  }
  *best_depth = bd;
  return best;
}

void set_entry(higgs_prefix_cache* pc, Node& n, const std::vector<int32_t>& pages) {
  if (n.cached) pool_release(pc->pool, n.pages);
  pool_retain(pc->pool, pages);
  n.cached = true;
  n.pages = pages;
  n.last_access = ++pc->clock;
}

// returns true if a new entry was created (prompt_cache.rs insert)
bool insert(higgs_prefix_cache* pc, Node& node, const int32_t* tok, int len, int pos,
            const std::vector<int32_t>& pages) {
  if (pos >= len) {
    const bool is_new = !node.cached;
    set_entry(pc, node, pages);
    return is_new;
  }
  const int32_t key = tok[pos];
  auto it = node.children.find(key);
  if (it == node.children.end()) {
    auto leaf = std::make_unique<Node>();
    leaf->edge.assign(tok + pos, tok + len);
    set_entry(pc, *leaf, pages);
    node.children[key] = std::move(leaf);
    return true;
  }
  Node& child = *it->second;
  int common = 0;
  while (common < (int)child.edge.size() && pos + common < len && child.edge[common] == tok[pos + common])
    ++common;
  if (common == (int)child.edge.size()) return insert(pc, child, tok, len, pos + common, pages);
  // split the edge at `common`
  std::unique_ptr<Node> old = std::move(it->second);
  node.children.erase(it);
  auto split = std::make_unique<Node>();
  split->edge.assign(old->edge.begin(), old->edge.begin() + common);
  old->edge.erase(old->edge.begin(), old->edge.begin() + common);
  const int32_t old_key = old->edge[0];
  split->children[old_key] = std::move(old);
  bool created;
  if (pos + common >= len) {
    set_entry(pc, *split, pages);
    created = true;
  } else {
    auto leaf = std::make_unique<Node>();
    leaf->edge.assign(tok + pos + common, tok + len);
    set_entry(pc, *leaf, pages);
    const int32_t nk = leaf->edge[0];
    split->children[nk] = std::move(leaf);
    created = true;
  }
  node.children[key] = std::move(split);
  return created;
}

bool oldest(const Node& n, uint64_t* t) {
  bool any = false;
  if (n.cached) {
    *t = n.last_access;
    any = true;
  }
  for (auto& kv : n.children) {
    uint64_t ct;
    if (oldest(*kv.second, &ct) && (!any || ct < *t)) {
      *t = ct;
      any = true;
    }
  }
  return any;
}

bool remove_with_time(higgs_prefix_cache* pc, Node& n, uint64_t t) {
  if (n.cached && n.last_access == t) {
    pool_release(pc->pool, n.pages);
    n.cached = false;
    n.pages.clear();
    return true;
  }
  for (auto& kv : n.children)
    if (remove_with_time(pc, *kv.second, t)) return true;
  return false;
}

void prune(Node& n, bool is_root) {
  for (auto& kv : n.children) prune(*kv.second, false);
  for (auto it = n.children.begin(); it != n.children.end();) {
    if (!it->second->cached && it->second->children.empty())
      it = n.children.erase(it);
    else
      ++it;
  }
  if (!is_root && !n.cached && n.children.size() == 1 && !n.edge.empty()) {
    std::unique_ptr<Node> only = std::move(n.children.begin()->second);
    n.children.clear();
    n.edge.insert(n.edge.end(), only->edge.begin(), only->edge.end());
    n.cached = only->cached;
    n.pages = std::move(only->pages);
    n.last_access = only->last_access;
    n.children = std::move(only->children);
  }
}

void release_all(higgs_prefix_cache* pc, Node& n) {
  if (n.cached) pool_release(pc->pool, n.pages);
  n.cached = false;
  n.pages.clear();
  for (auto& kv : n.children) release_all(pc, *kv.second);
  n.children.clear();
}

}  // namespace

// ---------------------------------------------------------------------------
// block pool
// ---------------------------------------------------------------------------
extern "C" int higgs_block_pool_create(int64_t num_pages, higgs_block_pool** out) {
  if (!out || num_pages <= 0 || num_pages > INT32_MAX)
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_block_pool_create: bad argument");
  auto* p = new higgs_block_pool;
  p->refcount.assign((size_t)num_pages, 0);
  p->free_list.reserve((size_t)num_pages);
  for (int64_t i = num_pages - 1; i >= 0; --i) p->free_list.push_back((int32_t)i);
  *out = p;
  return HIGGS_OK;
}

extern "C" int higgs_block_pool_destroy(higgs_block_pool* p) {
  delete p;
  return HIGGS_OK;
}

extern "C" int64_t higgs_block_pool_num_free(const higgs_block_pool* p) {
  return p ? (int64_t)p->free_list.size() : -1;
}

extern "C" int higgs_block_pool_alloc(higgs_block_pool* p, int n, int32_t* pages) {
  if (!p || n < 0 || (n > 0 && !pages)) return fail(HIGGS_ERR_INVALID_ARG, "higgs_block_pool_alloc: bad argument");
  if ((size_t)n > p->free_list.size())
    return fail(HIGGS_ERR_OUT_OF_PAGES, "higgs_block_pool_alloc: " + std::to_string(n) +
                                            " pages requested, " + std::to_string(p->free_list.size()) +
                                            " free");
  for (int i = 0; i < n; ++i) {
    const int32_t pg = p->free_list.back();
    p->free_list.pop_back();
    p->refcount[pg] = 1;
    pages[i] = pg;
  }
  return HIGGS_OK;
}

static int check_pages(const higgs_block_pool* p, const int32_t* pages, int n, const char* fn) {
  if (!p || n < 0 || (n > 0 && !pages)) return fail(HIGGS_ERR_INVALID_ARG, std::string(fn) + ": bad argument");
  for (int i = 0; i < n; ++i)
    if (pages[i] < 0 || pages[i] >= (int32_t)p->refcount.size() || p->refcount[pages[i]] <= 0)
      return fail(HIGGS_ERR_INVALID_ARG, std::string(fn) + ": page " + std::to_string(pages[i]) +
                                             " is not allocated");
  return HIGGS_OK;
}

extern "C" int higgs_block_pool_retain(higgs_block_pool* p, const int32_t* pages, int n) {
  int rc = check_pages(p, pages, n, "higgs_block_pool_retain");
  if (rc) return rc;
  for (int i = 0; i < n; ++i) p->refcount[pages[i]]++;
  return HIGGS_OK;
}

extern "C" int higgs_block_pool_release(higgs_block_pool* p, const int32_t* pages, int n) {
  int rc = check_pages(p, pages, n, "higgs_block_pool_release");
  if (rc) return rc;
  pool_release(p, std::vector<int32_t>(pages, pages + n));
  return HIGGS_OK;
}

extern "C" int higgs_block_pool_refcount(const higgs_block_pool* p, int32_t page) {
  if (!p || page < 0 || page >= (int32_t)p->refcount.size()) return -1;
  return p->refcount[page];
}

// ---------------------------------------------------------------------------
// prefix cache
// ---------------------------------------------------------------------------
extern "C" int higgs_prefix_cache_create(higgs_block_pool* pool, int max_entries,
                                         higgs_prefix_cache** out) {
  if (!pool || !out || max_entries < 0)
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_prefix_cache_create: bad argument");
  auto* pc = new higgs_prefix_cache;
  pc->pool = pool;
  pc->max_cached = max_entries;
  *out = pc;
  return HIGGS_OK;
}

extern "C" int higgs_prefix_cache_destroy(higgs_prefix_cache* pc) {
  if (!pc) return HIGGS_OK;
  release_all(pc, pc->root);
  delete pc;
  return HIGGS_OK;
}

extern "C" int higgs_prefix_cache_len(const higgs_prefix_cache* pc) { return pc ? pc->num_cached : -1; }

extern "C" int higgs_prefix_cache_clear(higgs_prefix_cache* pc) {
  if (!pc) return fail(HIGGS_ERR_INVALID_ARG, "higgs_prefix_cache_clear: null cache");
  release_all(pc, pc->root);
  pc->num_cached = 0;
  return HIGGS_OK;
}

extern "C" int higgs_prefix_cache_lookup(higgs_prefix_cache* pc, const int32_t* tokens, int n,
                                         int32_t* pages_out, int max_pages, int* matched_tokens) {
  if (!pc || (n > 0 && !tokens) || !matched_tokens || max_pages < 0 || (max_pages > 0 && !pages_out))
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_prefix_cache_lookup: bad argument");
  *matched_tokens = 0;
  int depth = 0;
  const Node* hit = find_deepest(pc->root, tokens, n, 0, &depth);
  if (!hit || depth < kMinPrefix) return HIGGS_OK;
  const int np = depth / kPage;
  if (np > max_pages)
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_prefix_cache_lookup: pages_out holds " +
                                           std::to_string(max_pages) + ", match needs " + std::to_string(np));
  const_cast<Node*>(hit)->last_access = ++pc->clock;
  std::vector<int32_t> used(hit->pages.begin(), hit->pages.begin() + np);
  for (int i = 0; i < np; ++i) pages_out[i] = used[i];
  pool_retain(pc->pool, used);  // the caller's reference
  *matched_tokens = depth;
  return HIGGS_OK;
}

extern "C" int higgs_prefix_cache_store(higgs_prefix_cache* pc, const int32_t* tokens, int n,
                                        const int32_t* pages, int n_pages) {
  if (!pc || n < 0 || (n > 0 && !tokens) || n_pages < 0 || (n_pages > 0 && !pages))
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_prefix_cache_store: bad argument");
  if (pc->max_cached == 0) return HIGGS_OK;
  const int full = (n / kPage) * kPage;  // only whole, immutable pages are shared
  if (full < kMinPrefix) return HIGGS_OK;
  const int need = full / kPage;
  if (n_pages < need)
    return fail(HIGGS_ERR_INVALID_ARG, "higgs_prefix_cache_store: " + std::to_string(need) +
                                           " pages needed for " + std::to_string(full) + " tokens");
  int rc = check_pages(pc->pool, pages, need, "higgs_prefix_cache_store");
  if (rc) return rc;
  std::vector<int32_t> pv(pages, pages + need);
  if (insert(pc, pc->root, tokens, full, 0, pv)) {
    pc->num_cached++;
    while (pc->num_cached > pc->max_cached) {
      uint64_t t;
      if (!oldest(pc->root, &t) || !remove_with_time(pc, pc->root, t)) break;
      pc->num_cached--;
      prune(pc->root, true);
    }
  }
  return HIGGS_OK;
}
