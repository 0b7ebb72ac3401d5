// Prints the team kernel's split of one launch (sk_split, then sk_warp_range for every CTA and
// warp), so a CPU test can check it on the real code:
//   split_check NB NTILES GRID WARPS  ->  "k teams" then one line per (cta, warp):
//                                         cta warp team wi leader t_lo t_hi b_lo b_hi
#include <cstdio>
#include <cstdlib>

#include "mv_streamk.cuh"

int main(int argc, char** argv) {
    if (argc < 5) return 2;
    laic::MvParams p{};
    p.nb = std::atoi(argv[1]);
    p.ntiles = std::atoi(argv[2]);
    const int grid = std::atoi(argv[3]), w = std::atoi(argv[4]);
    laic::sk_split(p, grid, w);
    std::printf("%d %d\n", p.team_k, p.team_n);
    for (int cta = 0; cta < grid; ++cta)
        for (int warp = 0; warp < w; ++warp) {
            const laic::SkWarpRange r = laic::sk_warp_range(p, cta, warp);
            std::printf("%d %d %d %d %d %d %d %d %d\n", cta, warp, r.team, r.wi, r.leader, r.t_lo, r.t_hi, r.b_lo,
                        r.b_hi);
        }
    return 0;
}
