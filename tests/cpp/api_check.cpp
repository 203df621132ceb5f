// Exercises the drop-in C++ API the way a caller of the reference would
// (vk_symbiote/examples/basic_inference.cpp): ConfigManager, GGUFLoader, Tokenizer and,
// with --gpu, VulkanSymbioteEngine. Prints one JSON object on stdout.
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "vk_symbiote/ConfigManager.h"
#include "vk_symbiote/GGUFLoader.h"
#include "vk_symbiote/Tokenizer.h"
#include "vk_symbiote/VulkanSymbioteEngine.h"

using namespace vk_symbiote;

static std::string ids_json(const std::vector<uint32_t>& v) {
    std::string s = "[";
    for (size_t i = 0; i < v.size(); i++) s += (i ? "," : "") + std::to_string(v[i]);
    return s + "]";
}

int main(int argc, char** argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: api_check <model.gguf> <config.toml> [--gpu prompt_ids_csv n_new]\n");
        return 2;
    }
    const std::string model = argv[1], cfg = argv[2];
    ConfigManager& cm = ConfigManager::instance();
    const bool file_ok = cm.load_from_file(cfg);
    char a0[] = "prog", a1[] = "--ram-gb", a2[] = "12.5", a3[] = "--tp", a4[] = "1", a5[] = "--model";
    std::vector<char> mp(model.begin(), model.end());
    mp.push_back(0);
    char* av[] = {a0, a1, a2, a3, a4, a5, mp.data()};
    cm.load_from_args(7, av);

    GGUFLoader loader(model);
    const bool loaded = (bool)loader.load();
    const ModelConfig mc = loader.get_model_config();
    const GGUFTensorInfo* q = loader.get_tensor("blk.0.attn_q.weight");
    auto emb = loader.read_tensor_cached("output_norm.weight");
    Tokenizer tok;
    const auto enc = tok.encode("hi  there\n");
    const std::string dec = tok.decode({104, 105, 360});

    printf("{\"file_ok\":%d,\"vram_gb\":%.3f,\"vram_explicit\":%d,\"ram_gb\":%.3f,\"lookahead\":%u,\"fp16\":%d,"
           "\"tp\":%u,\"model_path_ok\":%d,\"custom\":\"%s\",\"loaded\":%d,\"layers\":%u,\"hidden\":%u,"
           "\"heads\":%u,\"kv_heads\":%u,\"ffn\":%u,\"vocab\":%u,\"head_dim\":%u,\"q_rows\":%llu,"
           "\"norm0\":%.3f,\"tensors\":%llu,\"encode\":%s,\"decode\":\"%s\"",
           file_ok, cm.memory().vram_budget_gb, cm.vram_budget_explicit(), cm.memory().ram_budget_gb,
           cm.memory().prefetch_lookahead, cm.performance().use_fp16_math, cm.parallel().tp_size,
           cm.model_path() == model, cm.get_string("custom", "name", "none").c_str(), loaded, mc.num_layers,
           mc.hidden_size, mc.num_attention_heads, mc.num_key_value_heads, mc.intermediate_size, mc.vocab_size,
           mc.head_dim, q ? (unsigned long long)q->dimensions[1] : 0ull, emb ? emb.value()[0] : -1.0f,
           (unsigned long long)loader.tensor_count(), ids_json(enc).c_str(), dec.c_str());

    if (argc >= 6 && !strcmp(argv[3], "--gpu")) {
        std::vector<uint32_t> prompt;
        for (char* t = strtok(argv[4], ","); t; t = strtok(nullptr, ",")) prompt.push_back((uint32_t)atoi(t));
        const uint32_t n = (uint32_t)atoi(argv[5]);
        DeviceOptions o;
        o.max_seq = 256;
        VulkanSymbioteEngine engine(model, o);
        const auto ids = engine.generate_ids(prompt, n);
        engine.clear_kv_cache();
        const std::string text = engine.generate("ab c", 8);
        const auto stats = engine.run_benchmark_detailed(2, 8, 2);
        const auto vram = engine.get_vram_stats();
        printf(",\"ids\":%s,\"generate_len\":%zu,\"generate_prefix_ok\":%d,\"bench_tok_s\":%.1f,"
               "\"kv_bytes\":%zu,\"vram_used\":%llu,\"tok_s_metric\":%.1f,\"gbps\":%.1f",
               ids_json(ids).c_str(), text.size(), text.rfind("ab c", 0) == 0, stats.avg_tokens_per_sec,
               engine.get_kv_cache_memory_usage(), (unsigned long long)vram.used_size,
               engine.get_performance_metrics().average_tokens_per_second,
               engine.get_performance_metrics().memory_bandwidth_gbps);
        bool threw = false;
        try {
            engine.generate_ids(prompt, 1000);
        } catch (const std::exception&) {
            threw = true;
        }
        printf(",\"overflow_throws\":%d", threw);
        // generate_text_batch decodes its prompts together (max_batch 3): same text as one at a time
        const std::vector<std::string> prompts = {"ab c", "xyz", "hello there b"};
        std::vector<std::string> one;
        for (const auto& p : prompts) one.push_back(engine.generate(p, 12));
        DeviceOptions ob = o;
        ob.max_batch = 3;
        VulkanSymbioteEngine batched(model, ob);
        const auto many = batched.generate_text_batch(prompts, 12);
        printf(",\"batch_equal\":%d", (int)(many == one));
    }
    printf("}\n");
    return 0;
}
