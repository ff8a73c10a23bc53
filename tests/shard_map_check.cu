// Host-side check of the sequence-sharding ownership map (tt_attn.cuh):
// for many tier layouts and world sizes, the ranks' local positions cover
// every dense slot and every packed token exactly once, the local numbering
// of each rank is a bijection onto what it owns, ownership follows the
// documented rule (slot j -> rank j % w, packed granule k -> rank k % w), and
// the ring slots' token ids are exactly [total - n2, total).  Built with nvcc
// as a host program by tests/test_shard_map_cpu.py (no GPU needed).
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../tritiercache_b200/csrc/tt_attn.cuh"

using namespace tt;

static unsigned long long rng_state = 88172645463325252ull;
static int rnd(int n) {  // xorshift64, [0, n)
    rng_state ^= rng_state << 13;
    rng_state ^= rng_state >> 7;
    rng_state ^= rng_state << 17;
    return (int)(rng_state % (unsigned long long)(n > 0 ? n : 1));
}

static int fail(const char* what, int w, const TierCounts& tc, int grp) {
    std::printf("FAIL %s: w=%d n0=%d n1=%d n2=%d head=%d R=%d nblk=%d grp=%d\n", what, w, tc.n0, tc.n1, tc.n2,
                tc.ring_head, tc.ring_size, tc.nblk, grp);
    return 1;
}

int main() {
    int cases = 0;
    for (int it = 0; it < 4000; ++it) {
        TierCounts tc;
        const int R = 1 + rnd(300);
        tc.ring_size = R;
        tc.n0 = rnd(5);
        tc.n1 = rnd(2000);
        const bool full = rnd(4) != 0;
        tc.n2 = full ? R : rnd(R + 1);
        tc.ring_head = full ? rnd(R) : 0;
        tc.nblk = rnd(700);
        tc.total = tc.n0 + tc.n1 + tc.n2 + tc.nblk * 16 + rnd(50) + 100000;
        const int grp = rnd(2) ? 16 : 32;
        const int w = 1 + rnd(8);
        const int D = tc.n0 + tc.n1 + tc.n2, P = tc.nblk * grp;
        std::vector<int> seen0(tc.n0, 0), seen1(tc.n1, 0), seen2(R, 0), seenp(P, 0);
        std::vector<int> seen_id(tc.n2, 0);
        int nd_sum = 0, np_sum = 0;
        for (int r = 0; r < w; ++r) {
            const ShardMap M = shard_map(tc, grp, r, w);
            nd_sum += M.nd;
            np_sum += M.np;
            for (int i = 0; i < M.nd; ++i) {
                int slot = -1;
                const int tier = dense_local_slot(tc, i, r, w, slot);
                if (tier == 0) {
                    if (slot < 0 || slot >= tc.n0 || seen0[slot]++) return fail("sink slot", w, tc, grp);
                    if (w > 1 && slot % w != r) return fail("sink owner", w, tc, grp);
                } else if (tier == 1) {
                    if (slot < 0 || slot >= tc.n1 || seen1[slot]++) return fail("heavy-hitter slot", w, tc, grp);
                    if (w > 1 && slot % w != r) return fail("heavy-hitter owner", w, tc, grp);
                } else {
                    if (slot < 0 || slot >= R || seen2[slot]++) return fail("ring slot", w, tc, grp);
                    if (w > 1 && slot % w != r) return fail("ring owner", w, tc, grp);
                    if (!full && slot >= tc.n2) return fail("ring slot past the filled part", w, tc, grp);
                    const long long id = ring_slot_id(tc, slot);
                    const long long q = id - ((long long)tc.total - tc.n2);
                    if (q < 0 || q >= tc.n2 || seen_id[q]++) return fail("ring token id", w, tc, grp);
                    if (w <= 1 && q != i - tc.n0 - tc.n1) return fail("logical ring order", w, tc, grp);
                }
            }
            for (int i = 0; i < M.np; ++i) {
                const int p = packed_global(i, r, w);
                if (p < 0 || p >= P || seenp[p]++) return fail("packed token", w, tc, grp);
                if (w > 1 && (p / kShardGran) % w != r) return fail("packed owner", w, tc, grp);
                if (w > 1 && i / kShardGran != p / kShardGran / w) return fail("granule order", w, tc, grp);
            }
        }
        if (nd_sum != D || np_sum != P) return fail("totals", w, tc, grp);
        for (int j = 0; j < tc.n0; ++j)
            if (!seen0[j]) return fail("sink not covered", w, tc, grp);
        for (int j = 0; j < tc.n1; ++j)
            if (!seen1[j]) return fail("heavy hitter not covered", w, tc, grp);
        for (int j = 0; j < tc.n2; ++j)
            if (!seen2[j]) return fail("ring not covered", w, tc, grp);
        for (int p = 0; p < P; ++p)
            if (!seenp[p]) return fail("packed token not covered", w, tc, grp);
        ++cases;
    }
    std::printf("ok %d layouts\n", cases);
    return 0;
}
