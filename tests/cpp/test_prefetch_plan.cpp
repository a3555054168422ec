// Unit test of the DWDP engine's prefetch planning (csrc/prefetch_plan.h), host only.
// Built and run by tests/test_prefetch_plan.py; exits non-zero on the first failed check.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <set>
#include <vector>

#include "prefetch_plan.h"

using dwdp_plan::Copy;
using dwdp_plan::Expert;

static int failures = 0;
#define CHECK(cond)                                                   \
  do {                                                                \
    if (!(cond)) {                                                    \
      std::fprintf(stderr, "%s:%d: CHECK(%s)\n", __FILE__, __LINE__, #cond); \
      ++failures;                                                     \
    }                                                                 \
  } while (0)

static const size_t MiB = size_t(1) << 20;

// Every byte of every expert is copied exactly once, to the matching staging byte.
static void check_cover(const std::vector<Expert>& remote, const std::vector<Copy>& plan) {
  size_t planned = 0, expected = 0;
  for (const Copy& c : plan) planned += c.bytes;
  for (const Expert& x : remote) expected += x.bytes;
  CHECK(planned == expected);
  for (const Expert& x : remote) {
    size_t covered = 0;
    for (const Copy& c : plan) {
      const char* lo = std::max(c.src, x.src);
      const char* hi = std::min(c.src + c.bytes, x.src + x.bytes);
      if (lo < hi) {
        CHECK(c.dst - c.src == x.dst - x.src);  // the overlap lands on the expert's staging bytes
        covered += (size_t)(hi - lo);
      }
    }
    CHECK(covered == x.bytes);
  }
  for (size_t i = 0; i < plan.size(); ++i)
    for (size_t j = i + 1; j < plan.size(); ++j)
      CHECK(plan[i].src + plan[i].bytes <= plan[j].src || plan[j].src + plan[j].bytes <= plan[i].src);
}

int main() {
  // owner memory (3 owners) and staging, laid out as the engine lays them out: each owner's
  // experts back to back in ascending id, staging slots in ascending id
  const size_t E = 12, bytes = 9 * MiB;  // 4 experts per owner
  std::vector<char> mem(3 * 4 * bytes), stage(E * bytes);
  std::vector<Expert> all;
  for (size_t e = 0; e < E; ++e) all.push_back(Expert{(int)(e / 4), mem.data() + e * bytes, stage.data() + e * bytes, bytes});
  // rank 1 receives the experts of owners 0 and 2
  std::vector<Expert> remote;
  for (const Expert& x : all)
    if (x.owner != 1) remote.push_back(x);

  // one copy per expert: owners interleaved, starting with the owner after rank 1 (owner 2)
  {
    const auto plan = dwdp_plan::plan_prefetch(remote, 1, 0, 0);
    check_cover(remote, plan);
    CHECK(plan.size() == 8);
    CHECK(plan[0].src == all[8].src && plan[1].src == all[0].src && plan[2].src == all[9].src);
    for (const Copy& c : plan) CHECK(c.bytes == bytes);
  }
  // 2 MiB slices: an expert's slices consecutive, ragged last slice (9 MiB = 4 x 2 + 1)
  {
    const auto plan = dwdp_plan::plan_prefetch(remote, 1, 2 * MiB, 64 * MiB);
    check_cover(remote, plan);
    CHECK(plan.size() == 8 * 5);
    CHECK(plan[0].src == all[8].src && plan[4].bytes == MiB && plan[5].src == all[0].src);
  }
  // coalesced: each owner's 4 contiguous experts (36 MiB) as one run, 16 MiB cap -> 3 equal pieces
  {
    const auto plan = dwdp_plan::plan_prefetch(remote, 1, 0, 16 * MiB);
    check_cover(remote, plan);
    CHECK(plan.size() == 6);
    CHECK(plan[0].src == all[8].src && plan[1].src == all[0].src);  // owners interleaved, owner 2 first
    for (const Copy& c : plan) CHECK(c.bytes <= 12 * MiB + 256 && c.bytes % 256 == 0);
  }
  // coalesced, large cap: one copy per owner
  {
    const auto plan = dwdp_plan::plan_prefetch(remote, 1, 0, 64 * MiB);
    check_cover(remote, plan);
    CHECK(plan.size() == 2 && plan[0].bytes == 4 * bytes);
  }
  // a gap in staging (experts 9 and 10 not adjacent there) splits the run
  {
    std::vector<Expert> r = remote;
    for (Expert& x : r)
      if (x.src == all[10].src || x.src == all[11].src) x.dst += MiB;  // experts 10, 11 shifted
    const auto plan = dwdp_plan::plan_prefetch(r, 1, 0, 64 * MiB);
    size_t planned = 0;
    for (const Copy& c : plan) planned += c.bytes;
    CHECK(planned == 8 * bytes);
    CHECK(plan.size() == 3);  // owner 2: [8, 9] and [10, 11]; owner 0: [0..3]
  }
  // a rank that owns nothing it needs: empty plan
  {
    const auto plan = dwdp_plan::plan_prefetch({}, 0, 0, 64 * MiB);
    CHECK(plan.empty());
  }
  if (failures == 0) std::printf("prefetch plan: all checks passed\n");
  return failures == 0 ? 0 : 1;
}
