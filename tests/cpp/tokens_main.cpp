// tokens_main.cpp -- a caller of the reference's IPA helpers (rokoko::chunk_ipa /
// to_tokens, src/rokoko.h:141-221): one IPA string per input line; per line it
// prints the chunk count, then per chunk " | <bytes> <n> <ids...>".
#include <cstdio>
#include <iostream>
#include <string>

#include "tokens.h"

int main() {
    std::string line;
    while (std::getline(std::cin, line)) {
        const auto chunks = rokoko::chunk_ipa(line);
        std::printf("%zu", chunks.size());
        for (const auto& c : chunks) {
            std::printf(" | %zu %zu", c.phonemes.size(), c.tokens.size());
            for (int t : c.tokens) std::printf(" %d", t);
        }
        std::printf("\n");
    }
    return 0;
}
