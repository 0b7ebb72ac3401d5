// Prints the activation-record offsets (rec_off) of the tile and wide kernels for a few batch
// sizes and block counts, so a CPU test can check the layout's invariants on the real code.
//   layout_check NB NSEQ   ->  one line per (block, part, sequence, group): offset
#include <cstdio>
#include <cstdlib>

#include "mma_matvec.cuh"

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    const int nb = std::atoi(argv[1]), nseq = std::atoi(argv[2]);
    for (int bl = 0; bl < nb; ++bl)
        for (int part = 0; part < 2; ++part)
            for (int s = 0; s < nseq; ++s)
                for (int c = 0; c < 4; ++c) std::printf("%zu\n", laic::rec_off(bl, part, nseq, s, c));
    return 0;
}
