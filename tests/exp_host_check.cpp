// Host build of voxwerk_b200/csrc/vw_libm_exp.h against the C library's exp (test infrastructure).
// Reads doubles from argv[1]; prints "<count> <mismatches>" and the first mismatching arguments.
#include <cmath>
#include <cstdio>
#include <vector>

#include "vw_libm_exp.h"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    std::vector<double> xs;
    double v;
    while (std::fread(&v, sizeof v, 1, f) == 1) xs.push_back(v);
    std::fclose(f);
    long bad = 0;
    for (double x : xs) {
        const double a = vw::libm_exp(x), b = std::exp(x);
        if (!(a == b || (a != a && b != b))) {
            if (bad < 5) std::printf("# x=%a ours=%a libc=%a\n", x, a, b);
            ++bad;
        }
    }
    std::printf("%zu %ld\n", xs.size(), bad);
    return 0;
}
