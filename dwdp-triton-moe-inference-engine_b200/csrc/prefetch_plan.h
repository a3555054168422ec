// Copy planning of the DWDP engine's prefetch: which byte ranges move, in which order.
// Host-only and free of CUDA so that it is unit-tested on the CPU (tests/cpp); the engine
// (engine.cpp, dwdp_engine_prefetch) issues the planned copies on its copy streams.
//
// Order: the owners are interleaved (one expert, or one piece, of each owner in turn) and
// every rank starts with the owner after itself, so copies running side by side read
// different peers and the ranks of a node do not all start on the first owner's memory.
// Granularity, in priority order:
//   slice > 0     every expert moves as `slice`-byte pieces (the reference's 2 MiB slices,
//                 communication/buffers.cu:94-134);
//   coalesce > 0  each run of an owner's experts that is contiguous both in the owner's
//                 memory and in staging moves as near-equal pieces of at most ~`coalesce`
//                 bytes (an owner's experts lie back to back on both sides);
//   otherwise     one copy per expert.
#pragma once

#include <algorithm>
#include <cstddef>
#include <map>
#include <vector>

namespace dwdp_plan {

struct Expert {
  int owner;        // device that holds the expert
  const char* src;  // the expert's bytes in the owner's memory
  char* dst;        // its staging slot
  size_t bytes;
};

struct Copy {
  const char* src;
  char* dst;
  size_t bytes;
};

// Per-owner lists (input order kept), owners after `self` first.
inline std::vector<std::vector<Expert>> owners_in_turn(const std::vector<Expert>& remote, int self) {
  std::map<int, std::vector<Expert>> by_owner;
  for (const Expert& x : remote) by_owner[x.owner].push_back(x);
  std::vector<std::vector<Expert>> out;
  for (auto it = by_owner.upper_bound(self); it != by_owner.end(); ++it) out.push_back(it->second);
  for (auto it = by_owner.begin(); it != by_owner.end() && it->first <= self; ++it) out.push_back(it->second);
  return out;
}

inline void interleave(const std::vector<std::vector<Copy>>& lists, std::vector<Copy>& out) {
  for (size_t k = 0;; ++k) {
    bool any = false;
    for (const auto& l : lists)
      if (k < l.size()) {
        out.push_back(l[k]);
        any = true;
      }
    if (!any) break;
  }
}

inline std::vector<Copy> plan_prefetch(const std::vector<Expert>& remote, int self, size_t slice, size_t coalesce) {
  const auto owners = owners_in_turn(remote, self);
  std::vector<std::vector<Copy>> lists;
  for (const auto& lst : owners) {
    std::vector<Copy> pieces;
    if (slice == 0 && coalesce > 0) {
      for (size_t i = 0; i < lst.size();) {
        const char* src = lst[i].src;
        char* dst = lst[i].dst;
        size_t bytes = lst[i].bytes;
        size_t j = i + 1;
        for (; j < lst.size() && lst[j].src == src + bytes && lst[j].dst == dst + bytes; ++j) bytes += lst[j].bytes;
        const size_t n = (bytes + coalesce - 1) / coalesce;  // equal pieces, none tiny
        const size_t step = ((bytes + n - 1) / n + 255) & ~(size_t)255;
        for (size_t off = 0; off < bytes; off += step) pieces.push_back(Copy{src + off, dst + off, std::min(step, bytes - off)});
        i = j;
      }
      lists.push_back(std::move(pieces));
    } else {
      // one list entry per expert (its slices stay together, in order)
      lists.emplace_back();
      for (const Expert& x : lst) {
        std::vector<Copy> one;
        const size_t step = slice > 0 ? slice : x.bytes;
        for (size_t off = 0; off < x.bytes; off += step)
          one.push_back(Copy{x.src + off, x.dst + off, std::min(step, x.bytes - off)});
        lists.back().insert(lists.back().end(), one.begin(), one.end());
      }
    }
  }
  std::vector<Copy> out;
  if (slice == 0 && coalesce > 0) {
    interleave(lists, out);
    return out;
  }
  // experts interleaved across owners (an expert's slices consecutive)
  std::vector<size_t> pos(owners.size(), 0), ex(owners.size(), 0);
  for (bool any = true; any;) {
    any = false;
    for (size_t o = 0; o < owners.size(); ++o) {
      if (ex[o] >= owners[o].size()) continue;
      const Expert& x = owners[o][ex[o]];
      const size_t step = slice > 0 ? slice : x.bytes;
      const size_t n = x.bytes == 0 ? 0 : (x.bytes + step - 1) / step;
      for (size_t k = 0; k < n; ++k) out.push_back(lists[o][pos[o] + k]);
      pos[o] += n;
      ++ex[o];
      any = true;
    }
  }
  return out;
}

}  // namespace dwdp_plan
