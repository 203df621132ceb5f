// Host-code fuzz driver, built with AddressSanitizer and UndefinedBehaviorSanitizer by
// tests/test_host_sanitizers.py (no GPU, no CUDA code): damaged copies of a GGUF file go through
// GGUFLoader (parse, model config, tensor lookup, host fp32 reads, mapped tensors),
// Tokenizer::from_gguf with random bytes to encode and random ids to decode, and random text
// goes through ConfigManager's file parser; random slices of random GGUF blocks are repacked into
// the device row layout (exactly sized buffers) and the pack planner gets random budgets. Prints
// "ok <files> <refused>" when every input
// returned; any memory error or undefined behaviour aborts the process with a report.
//
//   host_fuzz <model.gguf> <scratch dir> <seed> <iterations>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <random>
#include <string>
#include <vector>

#include "kernels.h"
#include "vk_symbiote/ConfigManager.h"
#include "vk_symbiote/GGUFLoader.h"
#include "vk_symbiote/NomadPack.h"
#include "vk_symbiote/Tokenizer.h"

using namespace vk_symbiote;

static void write_file(const std::string& path, const std::vector<unsigned char>& d) {
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    f.write(reinterpret_cast<const char*>(d.data()), (std::streamsize)d.size());
}

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: host_fuzz <model.gguf> <scratch dir> <seed> <iterations>\n");
        return 2;
    }
    std::ifstream in(argv[1], std::ios::binary);
    const std::vector<unsigned char> base((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    if (base.size() < 64) return 2;
    const std::string dir = argv[2];
    std::mt19937_64 rng(std::strtoull(argv[3], nullptr, 10));
    const int iters = std::atoi(argv[4]);
    const size_t head = std::min<size_t>(base.size(), 4096);  // header, metadata, tensor infos
    auto uni = [&](size_t n) { return (size_t)(rng() % (n ? n : 1)); };
    int refused = 0;
    for (int it = 0; it < iters; it++) {
        std::vector<unsigned char> d = base;
        const size_t mode = uni(10);
        if (mode < 7) {
            for (size_t k = 0, n = 1 + uni(5); k < n; k++) d[8 + uni(head - 8)] = (unsigned char)uni(256);
        } else if (mode < 9) {  // a count or length field set huge
            const size_t p = 8 + uni(head - 16);
            const uint64_t v[3] = {~0ull, 0x7fffffffull, 1ull << 40};
            const uint64_t x = v[uni(3)];
            for (int b = 0; b < 8; b++) d[p + b] = (unsigned char)(x >> (8 * b));
        } else {
            d.resize(uni(d.size()));
        }
        const std::string path = dir + "/fuzz.gguf";
        write_file(path, d);
        {
            GGUFLoader g(path);
            if (!g.load()) {
                refused++;
            } else {
                (void)g.generate_packs(g.get_model_config());
                for (const std::string& name : g.get_tensor_names()) {
                    const GGUFTensorInfo* t = g.get_tensor(name);
                    if (t && t->element_count() <= (1u << 20)) (void)g.read_tensor_data(*t);
                    (void)g.map_tensor(name);
                }
                (void)g.get_vocabulary().size();
            }
        }
        auto tok = Tokenizer::from_gguf(path);
        std::string text;
        for (size_t k = 0, n = uni(48); k < n; k++) text += (char)uni(256);
        const std::vector<uint32_t> ids = tok->encode(text);
        std::vector<uint32_t> rid;
        for (size_t k = 0, n = uni(16); k < n; k++) rid.push_back((uint32_t)uni(2 * tok->vocab_size() + 3));
        (void)tok->decode(ids);
        (void)tok->decode(rid);
        if (it % 4 == 0) {  // the config parser on random text (brackets, quotes, '=' and '#' likely)
            const char alphabet[] = "[]=#\"'\n .-_0123456789abcdefgmrvtuxyzAB\t";
            std::string cfg;
            for (size_t k = 0, n = uni(300); k < n; k++) cfg += alphabet[uni(sizeof(alphabet) - 1)];
            std::vector<unsigned char> c(cfg.begin(), cfg.end());
            write_file(dir + "/fuzz.toml", c);
            (void)ConfigManager::instance().load_from_file(dir + "/fuzz.toml");
            // and the command line: flags of the reference, values that do not parse, missing values
            static const char* const flags[] = {"--model", "--config", "--vram-gb", "--ram-gb", "-v", "--verbose",
                                                "--power-profile", "--benchmark", "--tp", "--device", "--disable-gpu",
                                                "1.5", "-3", "x", "", "99999999999999999999", "nan"};
            std::vector<std::string> args = {"prog"};
            for (size_t k = 0, n = uni(8); k < n; k++) args.push_back(flags[uni(sizeof(flags) / sizeof(flags[0]))]);
            std::vector<char*> av;
            for (auto& a : args) av.push_back(&a[0]);
            (void)ConfigManager::instance().load_from_args((int)av.size(), av.data());
        }
    }
    for (int it = 0; it < iters; it++) {  // repack and residency planning
        const int dts[4] = {VSL_Q8_0, VSL_Q4_0, VSL_Q4_1, VSL_F16};
        const int dt = dts[uni(4)];
        const size_t cols = 32 * (1 + uni(16)), rows = 1 + uni(6);
        const size_t bb = vsl::is_quant(dt) ? vsl::gguf_block_bytes(dt) : 2;
        std::vector<unsigned char> blocks(rows * (cols / 32) * bb);
        for (auto& x : blocks) x = (unsigned char)uni(256);
        const size_t row0 = uni(rows), nrows = 1 + uni(rows - row0);
        size_t col0 = 32 * uni(cols / 32 + 1), ncols = 32 * uni(cols / 32 + 1);
        if (uni(8) == 0) col0 += 1 + uni(31);  // misaligned: refused
        const size_t ld = vsl::is_quant(dt) ? vsl::weight_row_bytes(dt, ncols) + 16 * uni(2) : 64;
        std::vector<unsigned char> out(nrows * ld + 1);
        if (vsl::repack_gguf_rows(dt, blocks.data(), cols, row0, nrows, col0, ncols, out.data(), ld, (int)uni(2)))
            refused++;
        const uint64_t lb = rng() >> uni(64), fb = rng() >> uni(64), budget = rng() >> uni(64);
        const PackResidency r = NomadPackManager::plan(lb >> 20, (uint32_t)uni(200), fb >> 20, budget >> 20);
        if (r.feasible && r.resident_layers + r.streamed_layers > 200) return 3;
    }
    printf("ok %d %d\n", iters, refused);
    return 0;
}
