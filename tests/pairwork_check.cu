// pairwork_check.cu — host check of the CTA-pair work decomposition
// (PairWork, csrc/gemm_common.cuh) that the stream-K kernels rely on: built
// and run by tests/test_pairwork.py. For many (tiles, k-blocks per tile,
// pairs) it checks that
//   - every (tile, k-block) belongs to exactly one pair;
//   - whole-wave tiles come first, in the strided order of the non-split
//     kernels;
//   - a tile split between pairs has one head (the segment holding its first
//     k-block), and the pairs the kernels' epilogue counts after it (the loop
//     over PairWork::split_start that both stream-K kernels run) are exactly
//     the pairs holding the rest of the tile;
//   - such a rest ("tail") is always its pair's first split segment, so a
//     head's wait for tails can never be part of a cycle.
#include <algorithm>
#include <cstdio>
#include <vector>

#include "gemm_common.cuh"

using lx2v::PairWork;

static int check(int n_tiles, int kb_per_tile, int npairs, bool whole_waves_first) {
    int fails = 0;
    std::vector<int> cover((size_t)n_tiles * kb_per_tile, 0);
    std::vector<int> head(n_tiles, -1), n_add(n_tiles, 0);
    std::vector<std::vector<int>> tails(n_tiles);
    const int dp = whole_waves_first ? (n_tiles / npairs) * npairs : 0;
    for (int pair = 0; pair < npairs; ++pair) {
        PairWork w;
        w.KB = kb_per_tile;
        w.pair = pair;
        w.npairs = npairs;
        w.sk = true;
        w.init_split(n_tiles, dp);
        const int n = w.count();
        long long total = 0;
        bool split_seen = false;
        for (int j = 0; j < n; ++j) {
            int t, kb0, kb1;
            w.seg(j, t, kb0, kb1);
            if (t < 0 || t >= n_tiles || kb0 < 0 || kb1 > kb_per_tile || kb0 >= kb1) {
                ++fails;
                continue;
            }
            for (int kb = kb0; kb < kb1; ++kb) cover[(size_t)t * kb_per_tile + kb]++;
            total += kb1 - kb0;
            if (j < w.my_dp) {
                if (kb0 != 0 || kb1 != kb_per_tile || t != pair + j * npairs) ++fails;
                continue;
            }
            if (kb0 > 0) {
                tails[t].push_back(pair);
                if (split_seen) ++fails;  // a tail must be the pair's first split segment
            } else if (kb1 < kb_per_tile) {
                if (head[t] >= 0) ++fails;
                head[t] = pair;
                const long long tile_end = (long long)(t + 1) * kb_per_tile;
                int a = 0;
                while (pair + 1 + a < npairs && w.split_start(n_tiles, pair + 1 + a) < tile_end) ++a;
                n_add[t] = a;
            }
            split_seen = true;
        }
        if (total != w.total_kb()) ++fails;
    }
    for (int c : cover)
        if (c != 1) ++fails;
    for (int t = 0; t < n_tiles; ++t) {
        if (head[t] < 0) {
            if (!tails[t].empty()) ++fails;  // a split tile without a head
            continue;
        }
        std::vector<int> want;
        for (int a = 1; a <= n_add[t]; ++a) want.push_back(head[t] + a);
        std::sort(tails[t].begin(), tails[t].end());
        if (tails[t] != want) ++fails;
    }
    return fails;
}

int main() {
    const int tiles[] = {1, 2, 5, 6, 13, 37, 73, 74, 75, 114, 148, 222, 245, 342, 665};
    const int kbs[] = {1, 2, 3, 11, 12, 24, 35, 70, 140};
    const int pairs[] = {1, 2, 3, 37, 74};
    int cases = 0, bad = 0;
    for (int t : tiles)
        for (int kb : kbs)
            for (int p : pairs)
                for (int hybrid = 0; hybrid < 2; ++hybrid) {
                    if ((long long)t * kb < p) continue;  // the hosts never split below one k-block per pair
                    ++cases;
                    const int f = check(t, kb, p, hybrid != 0);
                    if (f) {
                        ++bad;
                        std::printf("FAIL tiles=%d kb=%d pairs=%d whole_waves_first=%d: %d violations\n", t, kb, p,
                                    hybrid, f);
                    }
                }
    std::printf("%d cases, %d failing\n", cases, bad);
    return bad ? 1 : 0;
}
