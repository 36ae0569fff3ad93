// The round planner of the strict MSE's ordered walk (strict_mse.cu, mse_walk): which maps one
// round of the walk loads, in walk order.  Plain C++ that also compiles for the device, so that a
// host program can check it (tests/walk_plan_check.cpp).
//
// The walk summarises its input at three levels: a chunk map covers one chunk of elements, a block
// map 64 chunks, a superblock map 64 blocks.  One round covers up to `cap` consecutive maps from
// the walk's position on, each at the coarsest level its position allows: chunk maps up to the
// next block boundary, block maps up to the next superblock boundary, superblock maps, and, in
// front of a stop that is not the end of the segment, block maps and chunk maps again.  A map that
// failed (its state left the binade, or it cannot be used) is replaced by its children.  So a run
// that crosses a binade inside a superblock needs one round at each level going down and a single
// round back up.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define PCU_HOST_DEVICE __host__ __device__
#define PCU_UNROLL _Pragma("unroll")
#else
#define PCU_HOST_DEVICE
#define PCU_UNROLL
#endif

namespace pcu {

constexpr int kPlanLevels = 3;  // chunk, block, superblock; a parent map has 64 children
constexpr int kPlanRuns = 5;    // at most two runs going up and three coming down

// Each run of one level is one entry: maps first .. first + (start[e + 1] - start[e]) - 1 of
// `level`; a round's map j belongs to the entry e with start[e] <= j < start[e + 1].
struct WalkPlan {
    uint64_t first[kPlanRuns];
    unsigned start[kPlanRuns + 1];
    int level[kPlanRuns];
    int runs;
};

// Positions are in chunks; `c` is the walk's position.  `lim[l]`: the maps of level l lie wholly
// in front of the stop (at the end of the segment the last map of a level, which ends at the
// segment's end, counts).  The map of level `fail_level` at `fail_c` failed: every map inside it
// is of a finer level.  At most `cap` maps.
PCU_HOST_DEVICE inline void plan_walk_round(uint64_t c, const uint64_t lim[kPlanLevels], uint64_t fail_c,
                                            int fail_level, unsigned cap, WalkPlan &w) {
    unsigned total = 0;
    w.runs = 0;
    auto emit = [&](int l, uint64_t first, uint64_t end) {
        if (end > first && total < cap) {
            const uint64_t room = cap - total;
            w.first[w.runs] = first;
            w.level[w.runs] = l;
            w.start[w.runs] = total;
            total += (unsigned)(end - first < room ? end - first : room);
            ++w.runs;
        }
    };
    // up: finer maps until the next coarser map can be used
    uint64_t p = c;
    int top = kPlanLevels - 1;
    PCU_UNROLL
    for (int l = 0; l + 1 < kPlanLevels; ++l) {
        if (top < kPlanLevels - 1) break;
        const int sh = 6 * l, sh1 = 6 * (l + 1);
        uint64_t q = ((p + (1ull << sh1) - 1) >> sh1) << sh1;  // the next level-(l+1) boundary
        if (q == p && p == fail_c && fail_level == l + 1) q = p + (1ull << sh1);
        if ((q >> sh1) >= lim[l + 1]) {
            top = l;  // no coarser map from q on
        } else {
            emit(l, p >> sh, q >> sh);
            p = q;
        }
    }
    // down: each level up to its limit, then the finer ones in front of the stop
    PCU_UNROLL
    for (int l = kPlanLevels - 1; l >= 0; --l) {
        if (l > top) continue;
        emit(l, p >> (6 * l), lim[l]);
        const uint64_t e = lim[l] << (6 * l);
        if (e > p) p = e;
    }
    w.start[w.runs] = total;
}

}  // namespace pcu
