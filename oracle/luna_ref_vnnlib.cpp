// luna_ref_vnnlib.cpp -- test infrastructure, not product code.
//
// Prints Luna's own reading of a VNN-LIB property (luna_ref_vnnlib_parse in
// luna_ref_driver.cpp, i.e. VnnLibInputParser + OutputConstraintSet::toCMatrix
// compiled from the reference sources) as one JSON object, every float as a
// C99 hex literal so it round-trips exactly.  It runs as its own process:
// Luna's tokenizer uses std::regex, which crashes inside a Python process that
// has imported torch.
//
//   luna_ref_vnnlib <file.vnnlib> <n_in> <n_out> [<file> <n_in> <n_out> ...]
//
// One JSON line per property, in order.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

extern "C" int luna_ref_vnnlib_parse(const char* path, int64_t n_in, int64_t n_out, float* lower, float* upper,
                                     int64_t cap_rows, float* C, float* thresholds, int32_t* branch, int64_t* nspec,
                                     int32_t* n_branches, int32_t* spec_dropped, char* err, size_t errlen);

static void put_floats(const char* name, const float* p, size_t n) {
    std::printf("\"%s\": [", name);
    for (size_t k = 0; k < n; ++k) std::printf("%s\"%a\"", k ? ", " : "", (double)p[k]);
    std::printf("], ");
}

static std::string escaped(const char* s) {
    std::string o;
    for (; *s; ++s) {
        if (*s == '"' || *s == '\\') o += '\\';
        if ((unsigned char)*s < 0x20) continue;
        o += *s;
    }
    return o;
}

static void one(const char* path, int64_t n_in, int64_t n_out);

int main(int argc, char** argv) {
    if (argc < 4 || (argc - 1) % 3 != 0) {
        std::fprintf(stderr, "usage: %s <file.vnnlib> <n_in> <n_out> [...]\n", argv[0]);
        return 64;
    }
    for (int a = 1; a + 2 < argc; a += 3) one(argv[a], std::atoll(argv[a + 1]), std::atoll(argv[a + 2]));
    return 0;
}

static void one(const char* path, int64_t n_in, int64_t n_out) {
    std::vector<float> lo(n_in), hi(n_in);
    int64_t cap = 64, nspec = 0;
    int32_t nb = 0, dropped = 0;
    std::vector<float> C, thr;
    std::vector<int32_t> br;
    char err[4096] = {0};
    int rc;
    while (true) {
        C.assign((size_t)(cap * n_out), 0.f);
        thr.assign((size_t)cap, 0.f);
        br.assign((size_t)cap, 0);
        rc = luna_ref_vnnlib_parse(path, n_in, n_out, lo.data(), hi.data(), cap, C.data(), thr.data(), br.data(),
                                   &nspec, &nb, &dropped, err, sizeof err);
        if (rc != 3) break;
        cap = nspec;
    }
    std::printf("{\"rc\": %d, ", rc);
    if (rc == 0) {
        put_floats("lower", lo.data(), lo.size());
        put_floats("upper", hi.data(), hi.size());
        put_floats("C", C.data(), (size_t)(nspec * n_out));
        put_floats("thresholds", thr.data(), (size_t)nspec);
        std::printf("\"branches\": [");
        for (int64_t k = 0; k < nspec; ++k) std::printf("%s%d", k ? ", " : "", br[(size_t)k]);
        std::printf("], \"nspec\": %lld, \"n_branches\": %d, \"spec_dropped\": %d, ", (long long)nspec, nb, dropped);
    }
    std::printf("\"error\": \"%s\"}\n", escaped(err).c_str());
    std::fflush(stdout);
}
