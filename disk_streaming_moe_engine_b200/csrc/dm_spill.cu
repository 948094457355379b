// dm_spill.cu — residency policy of the expert cache when the expert pool spills to host
// memory (host code only).
//
// With expert_cache_slots = C > 0 a context keeps C expert records per layer in HBM (plus
// the shared expert, always resident) and all E records per layer in pinned host memory.
// Each batched step resolves, per layer, the experts its rows selected before the expert
// kernels run: hits refresh their recency, misses take a free slot or evict the least
// recently used unpinned slot not needed by this step, and are copied host -> HBM on the
// context stream.  The contract follows the reference's expert cache
// (src/io/lru_cache.mojo:225-610): begin_access counts a hit or claims a miss, a load
// evicts the resident unpinned entry with the oldest timestamp, pinned entries stay, and
// pinning is admitted only while the pinned total stays within 25 % of the capacity
// (finish_load :416-484; over budget the expert is kept unpinned).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <utility>
#include <vector>

#include "dismoen_cuda.h"
#include "dm_internal.h"

namespace dm {

void SpillPolicy::init(int L_, int E_, int C_) {
    L = L_;
    E = E_;
    C = C_;
    clock = 0;
    slot_of.assign(static_cast<size_t>(L) * E, -1);
    expert_in.assign(static_cast<size_t>(L) * C, -1);
    stamp.assign(static_cast<size_t>(L) * C, 0);
    pinned.assign(static_cast<size_t>(L) * C, 0);
    in_use.assign(static_cast<size_t>(C), 0);
    pinned_count.assign(L, 0);
    memset(stats, 0, sizeof stats);
}

// A free slot (lowest index) or the least recently used unpinned slot that this step does
// not use (ties to the lower slot); -1 when there is none.
int SpillPolicy::victim(int l) const {
    const int* ein = expert_in.data() + static_cast<size_t>(l) * C;
    for (int s = 0; s < C; ++s)
        if (ein[s] < 0 && !in_use[s]) return s;
    int best = -1;
    for (int s = 0; s < C; ++s) {
        if (in_use[s] || pinned[static_cast<size_t>(l) * C + s]) continue;
        if (best < 0 || stamp[static_cast<size_t>(l) * C + s] < stamp[static_cast<size_t>(l) * C + best]) best = s;
    }
    return best;
}

int SpillPolicy::place(int l, int e, std::vector<std::pair<int, int>>& loads) {
    const int s = victim(l);
    if (s < 0) return -1;
    int& old = expert_in[static_cast<size_t>(l) * C + s];
    if (old >= 0) {
        slot_of[static_cast<size_t>(l) * E + old] = -1;
        ++stats[3];  // eviction
    }
    old = e;
    slot_of[static_cast<size_t>(l) * E + e] = s;
    stamp[static_cast<size_t>(l) * C + s] = ++clock;
    in_use[s] = 1;
    loads.emplace_back(e, s);
    return s;
}

bool SpillPolicy::resolve(int l, const int* ids, int count, std::vector<std::pair<int, int>>& loads) {
    loads.clear();
    std::fill(in_use.begin(), in_use.end(), 0);
    // the distinct experts of the step, ascending
    std::vector<int> u(ids, ids + count);
    std::sort(u.begin(), u.end());
    u.erase(std::unique(u.begin(), u.end()), u.end());
    for (int e : u) {
        const int s = slot_of[static_cast<size_t>(l) * E + e];
        ++stats[0];
        if (s >= 0) {  // hit
            ++stats[1];
            stamp[static_cast<size_t>(l) * C + s] = ++clock;
            in_use[s] = 1;
        }
    }
    for (int e : u) {
        if (slot_of[static_cast<size_t>(l) * E + e] >= 0) continue;
        ++stats[2];  // miss
        if (place(l, e, loads) < 0) return false;
    }
    return true;
}

int SpillPolicy::pin(int l, int e, std::vector<std::pair<int, int>>& loads) {
    loads.clear();
    std::fill(in_use.begin(), in_use.end(), 0);
    int s = slot_of[static_cast<size_t>(l) * E + e];
    ++stats[0];  // a pin is an access: a hit when resident, else a miss that loads it
    if (s < 0) {
        ++stats[2];
        s = place(l, e, loads);
        if (s < 0) return -1;
    } else {
        ++stats[1];
    }
    uint8_t& p = pinned[static_cast<size_t>(l) * C + s];
    if (p) return 1;
    if (pinned_count[l] + 1 > C / 4) {  // the 25 % pin budget: kept unpinned
        ++stats[5];
        return 0;
    }
    p = 1;
    ++pinned_count[l];
    return 1;
}

}  // namespace dm

using namespace dm;

extern "C" int32_t dm_spill_simulate(int32_t L, int32_t E, int32_t C, int32_t steps, int32_t n, int32_t topk,
                                     const int32_t* ids, const int32_t* pins, int32_t npins, uint64_t* stats_out,
                                     int32_t* slot_of_out) {
    if (L <= 0 || E <= 0 || C <= 0 || C > E || steps < 0 || n <= 0 || topk <= 0 || (!ids && steps) || (npins && !pins))
        return DM_ERR_INVALID_ARG;
    SpillPolicy p;
    p.init(L, E, C);
    std::vector<std::pair<int, int>> loads;
    for (int i = 0; i < npins; ++i) {
        const int l = pins[2 * i], e = pins[2 * i + 1];
        if (l < 0 || l >= L || e < 0 || e >= E) return DM_ERR_INVALID_ARG;
        if (p.pin(l, e, loads) < 0) return DM_ERR_CAPACITY;
        p.stats[4] += loads.size();
    }
    for (int st = 0; st < steps; ++st)
        for (int l = 0; l < L; ++l) {
            const int32_t* row = ids + (static_cast<size_t>(st) * L + l) * n * topk;
            for (int i = 0; i < n * topk; ++i)
                if (row[i] < 0 || row[i] >= E) return DM_ERR_INVALID_ARG;
            if (!p.resolve(l, row, n * topk, loads)) return DM_ERR_CAPACITY;
            p.stats[4] += loads.size();
        }
    if (stats_out) memcpy(stats_out, p.stats, sizeof p.stats);
    if (slot_of_out) memcpy(slot_of_out, p.slot_of.data(), sizeof(int32_t) * p.slot_of.size());
    return DM_OK;
}
