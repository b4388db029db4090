// A caller written against the reference's model seam (its src/main.cu calls
// the same sequence: Weights::load, precompute_weight_norms, arenas sized with
// compute_decode_bytes, rokoko_infer, write_wav), compiled unchanged against
// include/rokoko/weights.h and linked with librokoko_compat.so.
//
//   rokoko_infer_main <weights.bin> <tokens.i32> <style.f32> <out.f32> [out.wav]
#include <cstdio>
#include <fstream>
#include <iterator>
#include <vector>

#include "weights.h"

template <typename T>
static std::vector<T> read_all(const char* path) {
    std::ifstream f(path, std::ios::binary);
    std::vector<char> b((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<T> out(b.size() / sizeof(T));
    std::copy(b.begin(), b.begin() + out.size() * sizeof(T), reinterpret_cast<char*>(out.data()));
    return out;
}

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s weights tokens style out [wav]\n", argv[0]);
        return 2;
    }
    std::vector<int> tokens = read_all<int>(argv[2]);
    std::vector<float> style = read_all<float>(argv[3]);
    if (style.size() != 256) return 2;
    cudaStream_t stream;
    cudaStreamCreate(&stream);
    rokoko::Weights w = rokoko::Weights::load(argv[1], stream);
    rokoko::precompute_weight_norms(w, stream);
    rokoko::GpuArena arena, decode_arena;
    arena.init(64 << 20);
    decode_arena.init(rokoko::compute_decode_bytes((int)tokens.size(), 32));
    const size_t ws_bytes = 16 << 20;
    float* d_ws = nullptr;
    cudaMalloc(&d_ws, ws_bytes);
    std::vector<float> audio = rokoko::rokoko_infer(w, tokens.data(), (int)tokens.size(), style.data(), stream,
                                                    arena, decode_arena, d_ws, ws_bytes);
    std::ofstream(argv[4], std::ios::binary).write(reinterpret_cast<const char*>(audio.data()),
                                                   (std::streamsize)(audio.size() * sizeof(float)));
    if (argc > 5 && !rokoko::write_wav(argv[5], audio.data(), (int)audio.size(), 24000)) return 1;
    fprintf(stderr, "%zu samples\n", audio.size());
    cudaFree(d_ws);
    arena.destroy();
    decode_arena.destroy();
    w.free();
    cudaStreamDestroy(stream);
    return 0;
}
