// Host check of the strict MSE walk's round planner (fusion-pcu_b200/csrc/mse_walk_plan.h), the
// same code the device walker runs.  For random segment sizes, stops, positions and failed maps it
// checks that a round's maps
//   * follow one another without a gap from the walk's position, in walk order;
//   * each lie wholly in front of the stop (at the segment's end, the last map of a level may be
//     partial);
//   * never include the failed map or another map of its level or coarser inside it;
//   * are each of the coarsest level the position allows;
//   * reach the stop (less than one chunk short of it) unless the round is full.
// Prints "walk plan ok" and exits 0, or prints the first failing case and exits 1.
#include <cstdio>
#include <cstdlib>

#include "mse_walk_plan.h"

namespace {

constexpr uint64_t kChunk = 1024;  // elements per chunk map (binary32)
constexpr unsigned kCap = 256;     // maps per round (the walker's threads)

uint64_t rng_state = 0x9e3779b97f4a7c15ull;
uint64_t next_u64() {  // xorshift64*
    rng_state ^= rng_state >> 12;
    rng_state ^= rng_state << 25;
    rng_state ^= rng_state >> 27;
    return rng_state * 0x2545f4914f6cdd1dull;
}
uint64_t below(uint64_t n) { return n ? next_u64() % n : 0; }

int fail(const char *what, uint64_t n, uint64_t stop, uint64_t c, uint64_t fail_c, int fail_level) {
    std::printf("FAIL %s: n=%llu stop=%llu chunk=%llu fail_c=%llu fail_level=%d\n", what, (unsigned long long)n,
                (unsigned long long)stop, (unsigned long long)c, (unsigned long long)fail_c, fail_level);
    return 1;
}

// One case: a segment of n elements, a stop (n, or the first fault in front of it), the walk at
// chunk c (c * kChunk < stop), and optionally the map of level fail_level at c failed.
int check(uint64_t n, uint64_t stop, uint64_t c, uint64_t fail_c, int fail_level) {
    const uint64_t count[3] = {(n + kChunk - 1) / kChunk, 0, 0};
    uint64_t cnt[3] = {count[0], (count[0] + 63) / 64, 0};
    cnt[2] = (cnt[1] + 63) / 64;
    const uint64_t lim[3] = {stop == n ? cnt[0] : stop / kChunk, stop == n ? cnt[1] : stop / (kChunk << 6),
                             stop == n ? cnt[2] : stop / (kChunk << 12)};
    pcu::WalkPlan w;
    pcu::plan_walk_round(c, lim, fail_c, fail_level, kCap, w);
    if (w.runs < 0 || w.runs > pcu::kPlanRuns || w.start[0] != 0) return fail("runs", n, stop, c, fail_c, fail_level);
    const unsigned total = w.start[w.runs];
    if (total > kCap) return fail("cap", n, stop, c, fail_c, fail_level);
    uint64_t pos = c;  // in chunks
    uint64_t end_elem = c * kChunk;
    for (int e = 0; e < w.runs; ++e) {
        if (w.start[e + 1] <= w.start[e]) return fail("empty run", n, stop, c, fail_c, fail_level);
        const int l = w.level[e];
        const uint64_t span = 1ull << (6 * l);  // chunks
        for (unsigned j = 0; j < w.start[e + 1] - w.start[e]; ++j) {
            const uint64_t idx = w.first[e] + j;
            if (idx * span != pos) return fail("gap or misaligned", n, stop, c, fail_c, fail_level);
            if (stop == n ? idx >= cnt[l] : (idx + 1) * span * kChunk > stop)
                return fail("past the stop", n, stop, c, fail_c, fail_level);
            if (fail_level < 3 && pos >= fail_c && pos < fail_c + (1ull << (6 * fail_level)) && l >= fail_level)
                return fail("the failed map again", n, stop, c, fail_c, fail_level);
            // coarsest: no coarser map that fits could start here
            for (int L = l + 1; L < 3; ++L) {
                const uint64_t sp = 1ull << (6 * L);
                const bool inside_failed =
                    fail_level < 3 && pos >= fail_c && pos < fail_c + (1ull << (6 * fail_level)) && L >= fail_level;
                if (pos % sp == 0 && (pos / sp) < lim[L] && !inside_failed)
                    return fail("a finer map where a coarser one fits", n, stop, c, fail_c, fail_level);
            }
            pos += span;
            end_elem = pos * kChunk < n ? pos * kChunk : n;
        }
    }
    if (total < kCap) {
        if (stop == n ? end_elem != n : stop - end_elem >= kChunk)
            return fail("short of the stop", n, stop, c, fail_c, fail_level);
    }
    return 0;
}

}  // namespace

int main() {
    const uint64_t sizes[] = {1, 1000, 1024, 1025, 65536, 65537, 4194304, 4194305, 1ull << 26, (1ull << 26) + 777,
                              (1ull << 28) + 3, 3 * 4194304 + 5000};
    for (int trial = 0; trial < 2000000; ++trial) {
        const int pick = (int)below(16);
        const uint64_t n = pick < 12 ? sizes[pick] : 1 + below(pick < 15 ? (1ull << 30) : (1ull << 44));
        const uint64_t stop = below(10) < 6 ? n : 1 + below(n);
        const uint64_t c = below((stop - 1) / kChunk + 1);
        if (c * kChunk >= stop) continue;
        uint64_t fail_c = ~0ull;
        int fail_level = 3;
        const int fl = (int)below(3);  // 0: none, 1: block, 2: superblock
        if (fl && c % (1ull << (6 * fl)) == 0) {
            fail_c = c;
            fail_level = fl;
        }
        if (check(n, stop, c, fail_c, fail_level)) return 1;
    }
    std::printf("walk plan ok\n");
    return 0;
}
