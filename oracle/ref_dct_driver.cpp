// ref_dct_driver.cpp -- harness that compiles the reference's own DCT matrix
// builders and eigenvalue-weight loop (host/density_scatter_ttnn_server_host.cpp
// lines 124-181 and 252-263, plain C++ with no TT-Metal dependency) where they
// lie in the reference tree, and dumps their outputs for golden fixtures.
// TEST INFRASTRUCTURE ONLY.  oracle/build_ref.sh extracts the two line ranges
// into oracle/_ref/*.inc at build time; nothing from the reference is committed.
//
// Usage: ref_dct M N bsx bsy out.bin
// out.bin = float32 arrays, in order: dct2(M), idct(M), idxst(M),
//           dct2(N), idct(N), idxst(N), wu(M*N), wv(M*N).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "ref_builders.inc"

static void ref_weights(int M, int N, float bsx, float bsy,
                        std::vector<float>& wu_out, std::vector<float>& wv_out) {
#include "ref_weights.inc"
    wu_out = wu_v;
    wv_out = wv_v;
}

static void put(FILE* f, const std::vector<float>& v) {
    fwrite(v.data(), sizeof(float), v.size(), f);
}

int main(int argc, char** argv) {
    if (argc != 6) {
        std::fprintf(stderr, "usage: %s M N bsx bsy out.bin\n", argv[0]);
        return 2;
    }
    int M = std::atoi(argv[1]), N = std::atoi(argv[2]);
    float bsx = (float)std::atof(argv[3]), bsy = (float)std::atof(argv[4]);
    FILE* f = std::fopen(argv[5], "wb");
    if (!f) return 1;
    put(f, build_dct2(M)); put(f, build_idct(M)); put(f, build_idxst(M));
    put(f, build_dct2(N)); put(f, build_idct(N)); put(f, build_idxst(N));
    std::vector<float> wu, wv;
    ref_weights(M, N, bsx, bsy, wu, wv);
    put(f, wu); put(f, wv);
    std::fclose(f);
    return 0;
}
