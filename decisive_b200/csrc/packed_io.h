// Host-side pieces of the packed checkpoint format (the reference's export_packed.rs:13-103): a
// small JSON reader/writer, SHA-256, and the manifest model.  Internal to libdecisive_b200.so.
#pragma once
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace dbio {

// ---- JSON (objects, arrays, strings, numbers, true/false/null; UTF-8 passed through)
struct Json {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;  // insertion order kept
    const Json* get(const std::string& key) const;  // nullptr when absent or not an object
};
bool json_parse(const std::string& text, Json* out, std::string* err);
std::string json_quote(const std::string& s);

// ---- SHA-256 (FIPS 180-4), lower-case hex digest
std::string sha256_hex(const uint8_t* data, size_t n);

// ---- manifest (packed-q4-e4.json / packed-q8-e8.json)
struct TensorEntry {
    std::string name;
    std::vector<int64_t> shape;
    uint64_t start = 0, end = 0;  // byte range inside the layer file
};
struct LayerEntry {
    std::string file;
    uint64_t bytes = 0;
    std::vector<TensorEntry> tensors;
    const TensorEntry* find_suffix(const std::string& suffix) const;
};
struct Manifest {
    int schema_version = 0;
    std::string revision, scheme;
    int group_size = 0, bits = 0;
    uint64_t group_bytes = 0, embedding_row_bytes = 0, decoder_bytes = 0;
    std::vector<LayerEntry> layers;
    std::string embedding, readout, norm;
    std::map<std::string, std::pair<uint64_t, std::string>> files;  // name -> (bytes, sha256)
};
bool read_manifest(const std::string& path, Manifest* m, std::string* err);
// Reads `dir/name`, checks its size against the manifest and, when verify, its SHA-256.
bool read_checked(const std::string& dir, const std::string& name, const Manifest& m, bool verify,
                  std::vector<uint8_t>* out, std::string* err);
bool write_file(const std::string& path, const void* data, size_t n, std::string* err);

}  // namespace dbio
