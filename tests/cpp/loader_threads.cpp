// Concurrency driver for the GGUF loader, built with ThreadSanitizer by
// tests/test_host_sanitizers.py (no GPU): four threads read every tensor through
// read_tensors_parallel (its own worker pool) and the LRU read_tensor_cached, while they also
// clear, resize and query the cache. Prints "ok <tensors>"; a data race aborts with a report.
//
//   loader_threads <model.gguf>
#include <cstdio>
#include <thread>
#include <vector>

#include "vk_symbiote/GGUFLoader.h"

using namespace vk_symbiote;

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    GGUFLoader g(argv[1]);
    if (!g.load()) {
        printf("load failed\n");
        return 1;
    }
    const std::vector<std::string> names = g.get_tensor_names();
    std::vector<std::thread> th;
    for (int t = 0; t < 4; t++)
        th.emplace_back([&, t] {
            for (int r = 0; r < 40; r++) {
                for (const auto& res : g.read_tensors_parallel(names))
                    if (!res) printf("read failed\n");
                for (const auto& n : names) (void)g.read_tensor_cached(n, r % 2 == 0);
                if (r % 8 == t) g.clear_tensor_cache();
                if (r % 16 == t) {
                    TensorCacheConfig c;
                    c.max_entries = 2 + (size_t)(r % 5);
                    g.configure_cache(c);
                }
                (void)g.get_tensor_cache_size();
            }
        });
    for (auto& x : th) x.join();
    printf("ok %zu\n", names.size());
    return 0;
}
