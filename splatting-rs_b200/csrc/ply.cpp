// The 3DGS binary PLY (instantsplat-rs/src/splat_ply.rs) to and from the packed parameter
// layout: include/splat_io.h states the format. Host code; device buffers cross in one
// cudaMemcpy each way.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "splat_constants.h"
#include "splat_io.h"

namespace {

thread_local std::string g_error;

sp_status fail(const std::string& message) {
    g_error = message;
    return SP_ERR_INVALID;
}

uint32_t stride_of(uint32_t sh_degree) { return SP_PARAM_STRIDE(sh_degree); }
uint32_t coefficients_of(uint32_t sh_degree) { return (sh_degree + 1) * (sh_degree + 1); }

struct FileCloser {
    void operator()(FILE* f) const {
        if (f) std::fclose(f);
    }
};
using File = std::unique_ptr<FILE, FileCloser>;

// Property names of a written file, in order.
std::vector<std::string> written_properties(uint32_t sh_degree) {
    std::vector<std::string> names = {"x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"};
    const uint32_t rest = 3 * (coefficients_of(sh_degree) - 1);
    for (uint32_t j = 0; j < rest; ++j) names.push_back("f_rest_" + std::to_string(j));
    for (const char* name : {"opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"})
        names.emplace_back(name);
    return names;
}

// One header line, without its end; false at end of file before any character.
bool read_line(FILE* f, std::string& line) {
    line.clear();
    int c;
    bool any = false;
    while ((c = std::fgetc(f)) != EOF) {
        any = true;
        line.push_back((char)c);
        if (c == '\n') break;
    }
    return any;
}

std::vector<std::string> words_of(const std::string& line) {
    std::vector<std::string> words;
    size_t i = 0;
    while (i < line.size()) {
        while (i < line.size() && std::isspace((unsigned char)line[i])) ++i;
        size_t j = i;
        while (j < line.size() && !std::isspace((unsigned char)line[j])) ++j;
        if (j > i) words.push_back(line.substr(i, j - i));
        i = j;
    }
    return words;
}

// Rust's {:?} of the line (quotes, \n and \" escaped) for the unexpected-line message.
std::string debug_quoted(const std::string& line) {
    std::string out = "\"";
    for (char c : line) {
        if (c == '\n') out += "\\n";
        else if (c == '\r') out += "\\r";
        else if (c == '\t') out += "\\t";
        else if (c == '"') out += "\\\"";
        else if (c == '\\') out += "\\\\";
        else out.push_back(c);
    }
    return out + "\"";
}

struct Header {
    uint64_t count = 0;
    std::vector<std::string> properties;
    uint32_t sh_degree = 0;
    long body = 0;  // byte offset of the first record
};

// parse_splat_ply's header loop (splat_ply.rs:56-82).
sp_status parse_header(FILE* f, const std::string& label, Header& h) {
    std::string line;
    if (!read_line(f, line)) return fail(label + ": not a PLY file");
    std::string first = line;
    while (!first.empty() && std::isspace((unsigned char)first.back())) first.pop_back();
    if (first != "ply") return fail(label + ": not a PLY file");
    bool have_count = false;
    for (;;) {
        if (!read_line(f, line)) return fail(label + ": header never ends");
        const std::vector<std::string> w = words_of(line);
        if ((w.size() == 3 && w[0] == "format" && w[1] == "binary_little_endian" && w[2] == "1.0") ||
            (!w.empty() && w[0] == "comment")) {
            continue;
        }
        if (w.size() == 3 && w[0] == "element") {
            if (w[1] != "vertex") return fail(label + ": unsupported element " + w[1]);
            char* end = nullptr;
            errno = 0;
            const unsigned long long n = std::strtoull(w[2].c_str(), &end, 10);
            if (errno || end == w[2].c_str() || *end || w[2][0] == '-' || w[2][0] == '+')
                return fail(label + ": vertex count " + w[2] + " is not a number");
            h.count = n;
            have_count = true;
            continue;
        }
        if (w.size() == 3 && w[0] == "property") {
            if (w[1] != "float") return fail(label + ": property " + w[2] + " is " + w[1] + ", not float");
            h.properties.push_back(w[2]);
            continue;
        }
        if (w.size() == 1 && w[0] == "end_header") break;
        return fail(label + ": unexpected header line " + debug_quoted(line));
    }
    if (!have_count) return fail("no vertex element");
    h.body = std::ftell(f);
    // The SH degree the f_rest_* properties carry.
    uint32_t rest = 0;
    for (const std::string& p : h.properties)
        if (p.rfind("f_rest_", 0) == 0) ++rest;
    h.sh_degree = 0;
    for (uint32_t d = 1; d <= 3; ++d)
        if (rest == 3 * (coefficients_of(d) - 1)) h.sh_degree = d;
    if (rest && !h.sh_degree)
        return fail(label + ": " + std::to_string(rest) + " f_rest properties are not an SH degree 1-3 layout");
    return SP_OK;
}

int column_of(const Header& h, const std::string& name) {
    for (size_t i = 0; i < h.properties.size(); ++i)
        if (h.properties[i] == name) return (int)i;
    return -1;
}

}  // namespace

extern "C" {

const char* sp_ply_error(void) { return g_error.c_str(); }

sp_status sp_ply_write(const char* path, const float* params, uint64_t count, uint32_t sh_degree,
                       int params_on_device) {
    if (!path || (!params && count)) return fail("null path or parameters");
    if (sh_degree > 3) return fail("SH degree above 3");
    const uint32_t stride = stride_of(sh_degree), k = coefficients_of(sh_degree);
    std::vector<float> staged;
    if (params_on_device && count) {
        staged.resize(count * stride);
        const cudaError_t err = cudaMemcpy(staged.data(), params, staged.size() * sizeof(float), cudaMemcpyDeviceToHost);
        if (err != cudaSuccess) {
            g_error = std::string("reading the parameters: ") + cudaGetErrorString(err);
            return err == cudaErrorMemoryAllocation ? SP_ERR_OUT_OF_MEMORY : SP_ERR_CUDA;
        }
        params = staged.data();
    }
    File f(std::fopen(path, "wb"));
    if (!f) return fail(std::string(path) + ": " + std::strerror(errno));
    // write_splat_ply_to (splat_ply.rs:22-46).
    const std::vector<std::string> names = written_properties(sh_degree);
    std::string header = "ply\nformat binary_little_endian 1.0\ncomment Exported from instantsplat-rs\nelement vertex " +
                         std::to_string(count) + "\n";
    for (const std::string& name : names) header += "property float " + name + "\n";
    header += "end_header\n";
    if (std::fwrite(header.data(), 1, header.size(), f.get()) != header.size()) return fail(std::string(path) + ": write failed");
    const size_t props = names.size();
    constexpr uint64_t kChunk = 1 << 15;
    std::vector<float> records(std::min<uint64_t>(count, kChunk) * props);
    for (uint64_t g0 = 0; g0 < count; g0 += kChunk) {
        const uint64_t here = std::min<uint64_t>(kChunk, count - g0);
        for (uint64_t i = 0; i < here; ++i) {
            const float* p = params + (g0 + i) * stride;
            float* r = records.data() + i * props;
            size_t o = 0;
            r[o++] = p[SP_SLOT_POSITION + 0];
            r[o++] = p[SP_SLOT_POSITION + 1];
            r[o++] = p[SP_SLOT_POSITION + 2];
            r[o++] = 0.0f;  // normals
            r[o++] = 0.0f;
            r[o++] = 0.0f;
            for (int c = 0; c < 3; ++c) r[o++] = p[SP_SLOT_SH + c];
            for (int c = 0; c < 3; ++c)
                for (uint32_t j = 1; j < k; ++j) r[o++] = p[SP_SLOT_SH + 3 * j + c];
            r[o++] = p[SP_SLOT_OPACITY];
            for (int a = 0; a < 3; ++a) r[o++] = p[SP_SLOT_LOG_SCALE + a];
            for (int a = 0; a < 4; ++a) r[o++] = p[SP_SLOT_ROTATION + a];
        }
        // Little-endian floats: the host's own layout on x86-64 and aarch64.
        if (std::fwrite(records.data(), sizeof(float) * props, here, f.get()) != here)
            return fail(std::string(path) + ": write failed");
    }
    if (std::fflush(f.get()) != 0) return fail(std::string(path) + ": write failed");
    return SP_OK;
}

sp_status sp_ply_read_header(const char* path, uint64_t* count, uint32_t* sh_degree) {
    if (!path || !count || !sh_degree) return fail("null argument");
    File f(std::fopen(path, "rb"));
    if (!f) return fail(std::string(path) + ": " + std::strerror(errno));
    Header h;
    const sp_status s = parse_header(f.get(), path, h);
    if (s != SP_OK) return s;
    *count = h.count;
    *sh_degree = h.sh_degree;
    return SP_OK;
}

sp_status sp_ply_read(const char* path, float* params, uint64_t count, uint32_t sh_degree, int params_on_device) {
    if (!path || (!params && count)) return fail("null path or parameters");
    if (sh_degree > 3) return fail("SH degree above 3");
    File f(std::fopen(path, "rb"));
    if (!f) return fail(std::string(path) + ": " + std::strerror(errno));
    const std::string label = path;
    Header h;
    sp_status s = parse_header(f.get(), label, h);
    if (s != SP_OK) return s;
    if (h.count != count)
        return fail(label + ": " + std::to_string(h.count) + " Gaussians, not " + std::to_string(count));
    // splat_ply.rs:83-94: the columns of the packed slots.
    static const char* const kNames[14] = {"x",       "y",       "z",       "f_dc_0", "f_dc_1", "f_dc_2", "opacity",
                                           "scale_0", "scale_1", "scale_2", "rot_0",  "rot_1",  "rot_2",  "rot_3"};
    static const int kSlots[14] = {SP_SLOT_POSITION,      SP_SLOT_POSITION + 1,  SP_SLOT_POSITION + 2,
                                   SP_SLOT_SH,            SP_SLOT_SH + 1,        SP_SLOT_SH + 2,
                                   SP_SLOT_OPACITY,       SP_SLOT_LOG_SCALE,     SP_SLOT_LOG_SCALE + 1,
                                   SP_SLOT_LOG_SCALE + 2, SP_SLOT_ROTATION,      SP_SLOT_ROTATION + 1,
                                   SP_SLOT_ROTATION + 2,  SP_SLOT_ROTATION + 3};
    const uint32_t stride = stride_of(sh_degree);
    std::vector<std::pair<int, int>> columns;  // (file column, packed slot)
    for (int i = 0; i < 14; ++i) {
        const int c = column_of(h, kNames[i]);
        if (c < 0) return fail(label + ": no property " + kNames[i]);
        columns.emplace_back(c, kSlots[i]);
    }
    const uint32_t k_file = coefficients_of(h.sh_degree), k_out = coefficients_of(sh_degree);
    for (uint32_t j = 1; j < k_out && j < k_file; ++j)
        for (int c = 0; c < 3; ++c) {
            const std::string name = "f_rest_" + std::to_string(c * (k_file - 1) + (j - 1));
            const int col = column_of(h, name);
            if (col < 0) return fail(label + ": no property " + name);
            columns.emplace_back(col, (int)(SP_SLOT_SH + 3 * j + c));
        }
    std::vector<float> host;
    float* out = params;
    if (params_on_device) {
        host.resize(count * stride);
        out = host.data();
    }
    const size_t props = h.properties.size();
    constexpr uint64_t kChunk = 1 << 15;
    std::vector<float> records(std::min<uint64_t>(count, kChunk) * props);
    for (uint64_t g0 = 0; g0 < count; g0 += kChunk) {
        const uint64_t here = std::min<uint64_t>(kChunk, count - g0);
        if (std::fread(records.data(), sizeof(float) * props, here, f.get()) != here)
            return fail(label + ": failed to fill whole buffer");
        for (uint64_t i = 0; i < here; ++i) {
            const float* r = records.data() + i * props;
            float* p = out + (g0 + i) * stride;
            std::memset(p, 0, stride * sizeof(float));
            for (const auto& column : columns) p[column.second] = r[column.first];
        }
    }
    if (params_on_device && count) {
        const cudaError_t err = cudaMemcpy(params, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (err != cudaSuccess) {
            g_error = std::string("writing the parameters: ") + cudaGetErrorString(err);
            return err == cudaErrorMemoryAllocation ? SP_ERR_OUT_OF_MEMORY : SP_ERR_CUDA;
        }
    }
    return SP_OK;
}

}  // extern "C"
