// host_io.h - model container reading on the host: safetensors shards and
// config.json, with the reference's discovery order and key semantics.
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/picchio_b200.h"

namespace pc {

enum StDtype { ST_F32, ST_F16, ST_BF16, ST_I32, ST_I16, ST_I8, ST_U8, ST_F64, ST_BOOL, ST_UNKNOWN };

struct StTensor {
    StDtype dtype = ST_UNKNOWN;
    std::vector<int64_t> shape;
    int64_t begin = 0, end = 0;  // absolute file offsets
    int file = -1;
    int64_t numel() const;
    int64_t nbytes() const { return end - begin; }
};

// Tensor database over several shard files; the first file that holds a
// name wins (st_find's linear search, st.h:356-362).
class StDB {
public:
    ~StDB();
    bool open_file(const std::string &path, std::string *err);
    const StTensor *find(const std::string &name) const;
    // Reads `bytes` bytes at `offset` inside the tensor.
    bool read(const StTensor &t, void *dst, int64_t bytes, int64_t offset = 0) const;
    int n_files() const { return (int)fds_.size(); }
    size_t n_tensors() const { return map_.size(); }

private:
    std::vector<int> fds_;
    std::unordered_map<std::string, StTensor> map_;
};

// Opens the shards of a model directory in picchio's order
// (picchio.c:2852-2912): dense.safetensors, model.safetensors,
// model-NNNNN-of-NNNNN.safetensors, the ';'-separated MODEL_AUX list,
// model-NNNNN.safetensors, experts-NN.safetensors.
bool open_model_dir(StDB &db, const std::string &dir, std::string *err);

// cfg_load (picchio.c:349-425) over json.h's key search: a key matches
// wherever '"key"' is followed by ':' (nested objects included).
bool load_config(const std::string &dir, pc_model_cfg *cfg, std::string *err);

}  // namespace pc
