// Host-side check of the sequence-sharding ownership map (tt_attn.cuh):
// for many tier layouts and world sizes, the ranks' local positions cover
// every dense slot and every packed token exactly once, the local numbering
// of each rank is a bijection onto what it owns, ownership follows the
// documented rule (slot j -> rank j % w, packed granule k -> rank k % w), and
// the ring slots' token ids are exactly [total - n2, total); and the float
// order keys behind the radix select and the routing rows' (score, slot)
// minimum keep float order.  Built with nvcc as a host program by
// tests/test_shard_map_cpu.py (no GPU needed).
#include <cstdio>
#include <cstdlib>
#include <cstring>
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
    // order keys (radix select, routing rows): key order is float order, the
    // round trip is exact, and the complemented (score, slot) keys of the
    // routing rows give the strict-< argmin with the first slot on ties
    const float probes[] = {-1e30f, -2.5f, -1.0f, -1e-30f, -0.0f, 0.0f, 1e-30f, 1e-7f, 0.25f, 1.0f, 3.5f, 1e30f};
    const int np_ = (int)(sizeof(probes) / sizeof(probes[0]));
    for (int a = 0; a < np_; ++a) {
        const float x = probes[a];
        const float y = key_value(order_key(x));
        if (memcmp(&x, &y, 4) != 0) { std::printf("FAIL key round trip %g\n", x); return 1; }
        for (int b = 0; b < np_; ++b) {
            const float z = probes[b];
            if ((x < z) != (order_key(x) < order_key(z)) && !(x == 0.0f && z == 0.0f)) {
                std::printf("FAIL key order %g %g\n", x, z);
                return 1;
            }
        }
    }
    for (int it = 0; it < 20000; ++it) {
        float v[4];
        int slot[4];
        for (int k = 0; k < 4; ++k) {
            v[k] = (float)rnd(8) * 0.125f;  // ties are common
            slot[k] = rnd(1000);
        }
        unsigned long long best = 0ull;  // complement, 0 = none
        int bi = -1;
        float bv = 0.f;
        for (int k = 0; k < 4; ++k) {
            const unsigned long long key = ~(((unsigned long long)order_key(v[k]) << 32) | (uint32_t)slot[k]);
            best = key > best ? key : best;
            if (bi < 0 || v[k] < bv || (v[k] == bv && slot[k] < bi)) { bv = v[k]; bi = slot[k]; }
        }
        const unsigned long long key = ~best;
        if (key_value((uint32_t)(key >> 32)) != bv || (int)(uint32_t)key != bi) {
            std::printf("FAIL routing minimum\n");
            return 1;
        }
    }
    std::printf("ok %d layouts\n", cases);
    return 0;
}
