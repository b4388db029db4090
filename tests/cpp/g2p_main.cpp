// g2p_main.cpp -- a caller written against the reference's phonemizer class
// (rokoko::G2PModelCuda, src/g2p.h:374-430): load a G2P3 file, phonemize each
// line of a UTF-8 text file, write one result per line.
//     g2p_main <model.bin> <texts.txt> <out.txt>
#include <cuda_runtime.h>

#include <cstdio>
#include <fstream>
#include <string>

#include "g2p.h"

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: g2p_main <model.bin> <texts.txt> <out.txt>\n");
        return 2;
    }
    cudaStream_t stream;
    if (cudaStreamCreate(&stream) != cudaSuccess) return 1;
    rokoko::G2PModelCuda model;
    if (!model.load(argv[1], stream)) {
        std::fprintf(stderr, "failed to load %s\n", argv[1]);
        return 1;
    }
    std::printf("params %zu bytes\n", model.param_bytes());
    std::ifstream in(argv[2]);
    std::ofstream out(argv[3]);
    std::string line;
    while (std::getline(in, line)) out << model.infer(line, stream) << "\n";
    model.free();
    cudaStreamDestroy(stream);
    return model.loaded() ? 1 : 0;
}
