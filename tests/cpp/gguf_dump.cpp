// gguf_dump.cpp -- test program: parse a GGUF file with hesa_gguf::File
// (hesa-llm_b200/backend/gguf_file.cpp) and print what it read as one JSON
// object, so tests/test_gguf.py can compare it with the file's writer (the
// independent gguf Python package). No GPU.
#include "backend/gguf_file.hpp"

#include <cstdio>
#include <string>

namespace {

std::string esc(const std::string& s) {
    std::string o;
    for (unsigned char c : s) {
        if (c == '"' || c == '\\') {
            o += '\\';
            o += static_cast<char>(c);
        } else if (c < 0x20) {
            char b[8];
            std::snprintf(b, sizeof(b), "\\u%04x", c);
            o += b;
        } else {
            o += static_cast<char>(c);
        }
    }
    return o;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: gguf_dump <file.gguf>\n");
        return 2;
    }
    hesa_gguf::File f;
    const int rc = f.open(argv[1]);
    std::printf("{\"rc\": %d, \"error\": \"%s\"", rc, esc(f.error()).c_str());
    if (rc != hesa_gguf::kOk) {
        std::printf("}\n");
        return 0;
    }
    std::printf(", \"version\": %u, \"alignment\": %llu, \"data_offset\": %llu, \"kv\": {", f.version(),
                static_cast<unsigned long long>(f.alignment()), static_cast<unsigned long long>(f.data_offset()));
    bool first = true;
    for (const auto& kv : f.metadata()) {
        const hesa_gguf::Value& v = kv.second;
        std::printf("%s\"%s\": {\"type\": %u", first ? "" : ", ", esc(kv.first).c_str(),
                    static_cast<unsigned>(v.type));
        first = false;
        if (v.is_int()) std::printf(", \"i\": %lld, \"u\": %llu", static_cast<long long>(v.i),
                                    static_cast<unsigned long long>(v.u));
        if (v.is_float()) std::printf(", \"f\": %.17g", v.f);
        if (v.type == hesa_gguf::ValueType::STRING) std::printf(", \"s\": \"%s\"", esc(v.s).c_str());
        if (v.type == hesa_gguf::ValueType::ARRAY) {
            std::printf(", \"elem\": %u, \"count\": %llu, \"ints\": [", static_cast<unsigned>(v.elem),
                        static_cast<unsigned long long>(v.count));
            for (size_t i = 0; i < v.ints.size(); ++i) std::printf("%s%lld", i ? ", " : "", static_cast<long long>(v.ints[i]));
            std::printf("], \"floats\": [");
            for (size_t i = 0; i < v.floats.size(); ++i) std::printf("%s%.17g", i ? ", " : "", v.floats[i]);
            std::printf("], \"strings\": [");
            for (size_t i = 0; i < v.strings.size(); ++i)
                std::printf("%s\"%s\"", i ? ", " : "", esc(v.strings[i]).c_str());
            std::printf("]");
        }
        std::printf("}");
    }
    std::printf("}, \"tensors\": [");
    for (size_t i = 0; i < f.tensors().size(); ++i) {
        const auto& t = f.tensors()[i];
        std::printf("%s{\"name\": \"%s\", \"type\": %u, \"ne\": [%lld, %lld, %lld, %lld], \"n_dims\": %u, "
                    "\"offset\": %llu, \"bytes\": %llu, \"file_offset\": %lld}",
                    i ? ", " : "", esc(t.name).c_str(), t.type, static_cast<long long>(t.ne[0]),
                    static_cast<long long>(t.ne[1]), static_cast<long long>(t.ne[2]), static_cast<long long>(t.ne[3]),
                    t.n_dims, static_cast<unsigned long long>(t.offset), static_cast<unsigned long long>(t.bytes),
                    t.data ? static_cast<long long>(f.data_offset() + t.offset) : -1LL);
    }
    std::printf("]");
    hesa_gguf::LlamaShape s;
    if (f.llama_shape(s) == hesa_gguf::kOk)
        std::printf(", \"llama\": {\"arch\": \"%s\", \"n_layer\": %lld, \"d_model\": %lld, \"n_head\": %lld, "
                    "\"n_kv_head\": %lld, \"d_ff\": %lld, \"vocab\": %lld, \"context\": %lld, \"rms_eps\": %.9g, "
                    "\"rope_base\": %.9g}",
                    esc(s.arch).c_str(), static_cast<long long>(s.n_layer), static_cast<long long>(s.d_model),
                    static_cast<long long>(s.n_head), static_cast<long long>(s.n_kv_head),
                    static_cast<long long>(s.d_ff), static_cast<long long>(s.vocab),
                    static_cast<long long>(s.context), s.rms_eps, s.rope_base);
    std::printf("}\n");
    return 0;
}
