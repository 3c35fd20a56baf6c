// gguf.cpp -- the GGUF container reader (include/styx_gguf.h).
//
// A restatement of Gguf::open (crates/gguf-rs/src/lib.rs:41-120) over a
// read-only memory mapping of the file: the same field order, limits,
// defaults and error messages.  Values are kept as a flat list of nodes;
// arrays of scalars store their elements inline.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/styx_gguf.h"

namespace styx {
int set_error(int code, const char *msg);
}

namespace {

constexpr uint32_t kMagic = 0x46554747u;             // "GGUF" little-endian (lib.rs:47)
constexpr uint64_t kMaxString = uint64_t(1) << 24;    // lib.rs:139
constexpr uint64_t kMaxArray = uint64_t(1) << 28;     // lib.rs:226
// Arrays of arrays nest by recursion; past this depth the file is refused
// (the reference recurses without a limit, so such a file exhausts its stack).
constexpr int kMaxDepth = 64;

struct Node {
    uint32_t type = 0;         // styx_gguf_vtype
    uint32_t elem = 0;         // arrays: element type
    uint64_t bits = 0;         // scalars: the value's bytes, zero-extended
    std::string str;           // strings
    std::vector<uint64_t> sc;  // arrays of scalars: element bits
    std::vector<uint64_t> kids;  // arrays of strings / arrays: node indices
    uint64_t count = 1;
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0, size = 0;
};

struct Error {
    int code;
    std::string msg;
};

// A bounds-checked little-endian cursor; running off the end is the
// reader's UnexpectedEof ("failed to fill whole buffer").
struct Cursor {
    const uint8_t *base, *p, *end;
    bool take(void *dst, size_t n, Error &e) {
        if (static_cast<size_t>(end - p) < n) {
            e = {STYX_EEOF, "failed to fill whole buffer"};
            return false;
        }
        std::memcpy(dst, p, n);
        p += n;
        return true;
    }
    template <class T>
    bool get(T &v, Error &e) {
        return take(&v, sizeof(T), e);   // the host is little-endian, as GGUF
    }
    uint64_t pos() const { return static_cast<uint64_t>(p - base); }
};

// Strict UTF-8 (the well-formed byte sequences of Unicode Table 3-7).
// On failure: the index where the bad sequence starts and its length, or
// length 0 when the input ends inside an otherwise valid sequence; reported
// as "invalid utf-8 sequence of N bytes from index I" / "incomplete utf-8
// byte sequence from index I".
bool utf8_ok(const uint8_t *s, size_t n, size_t &at, int &len) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        if (c < 0x80) {
            i++;
            continue;
        }
        int width = 0;
        if (c >= 0xC2 && c <= 0xDF) width = 2;
        else if (c >= 0xE0 && c <= 0xEF) width = 3;
        else if (c >= 0xF0 && c <= 0xF4) width = 4;
        at = i;
        if (width == 0) {
            len = 1;
            return false;
        }
        auto cont = [](uint8_t b) { return b >= 0x80 && b <= 0xBF; };
        // second byte: narrower ranges after E0, ED, F0 and F4
        if (i + 1 >= n) {
            len = 0;
            return false;
        }
        const uint8_t c1 = s[i + 1];
        bool second = cont(c1);
        if (c == 0xE0) second = c1 >= 0xA0 && c1 <= 0xBF;
        else if (c == 0xED) second = c1 >= 0x80 && c1 <= 0x9F;
        else if (c == 0xF0) second = c1 >= 0x90 && c1 <= 0xBF;
        else if (c == 0xF4) second = c1 >= 0x80 && c1 <= 0x8F;
        if (!second) {
            len = 1;
            return false;
        }
        for (int k = 2; k < width; k++) {
            if (i + k >= n) {
                len = 0;
                return false;
            }
            if (!cont(s[i + k])) {
                len = k;
                return false;
            }
        }
        i += width;
    }
    return true;
}

bool read_string(Cursor &c, std::string &out, Error &e) {
    uint64_t len;
    if (!c.get(len, e)) return false;
    if (len > kMaxString) {
        e = {STYX_EDATA, "String too long"};
        return false;
    }
    if (static_cast<uint64_t>(c.end - c.p) < len) {
        e = {STYX_EEOF, "failed to fill whole buffer"};
        return false;
    }
    size_t at = 0;
    int bad = 0;
    if (!utf8_ok(c.p, len, at, bad)) {
        char m[96];
        if (bad) std::snprintf(m, sizeof m, "Invalid UTF-8: invalid utf-8 sequence of %d bytes from index %zu", bad, at);
        else std::snprintf(m, sizeof m, "Invalid UTF-8: incomplete utf-8 byte sequence from index %zu", at);
        e = {STYX_EDATA, m};
        return false;
    }
    out.assign(reinterpret_cast<const char *>(c.p), len);
    c.p += len;
    return true;
}

// bytes of a scalar value type, 0 for string / array / unknown
int scalar_bytes(uint32_t t) {
    switch (t) {
    case STYX_GGUF_U8: case STYX_GGUF_I8: case STYX_GGUF_BOOL: return 1;
    case STYX_GGUF_U16: case STYX_GGUF_I16: return 2;
    case STYX_GGUF_U32: case STYX_GGUF_I32: case STYX_GGUF_F32: return 4;
    case STYX_GGUF_U64: case STYX_GGUF_I64: case STYX_GGUF_F64: return 8;
    default: return 0;
    }
}

Error unknown_type(uint32_t t) {
    char m[64];
    std::snprintf(m, sizeof m, "Unknown value type: %u", t);
    return {STYX_EDATA, m};
}

bool read_scalar(Cursor &c, uint32_t t, uint64_t &bits, Error &e) {
    const int nb = scalar_bytes(t);
    uint64_t v = 0;
    if (!c.take(&v, static_cast<size_t>(nb), e)) return false;
    if (t == STYX_GGUF_BOOL) v = v != 0;   // read_u8 != 0 (lib.rs:165)
    bits = v;
    return true;
}

// read_value (lib.rs:155-176) into nodes[idx]; arrays recurse (read_array,
// lib.rs:222-235): the element type is only checked when an element is read
bool read_value(Cursor &c, uint32_t t, std::vector<Node> &nodes, size_t idx, Error &e, int depth = 0) {
    if (depth > kMaxDepth) {
        e = {STYX_EDATA, "Array nesting too deep"};
        return false;
    }
    nodes[idx].type = t;
    nodes[idx].elem = t;
    if (scalar_bytes(t)) return read_scalar(c, t, nodes[idx].bits, e);
    if (t == STYX_GGUF_STRING) {
        std::string s;
        if (!read_string(c, s, e)) return false;
        nodes[idx].str = std::move(s);
        return true;
    }
    if (t != STYX_GGUF_ARRAY) {
        e = unknown_type(t);
        return false;
    }
    uint32_t et;
    uint64_t count;
    if (!c.get(et, e) || !c.get(count, e)) return false;
    if (count > kMaxArray) {
        e = {STYX_EDATA, "Array too long"};
        return false;
    }
    nodes[idx].elem = et;
    nodes[idx].count = count;
    if (count == 0) return true;
    if (scalar_bytes(et)) {
        std::vector<uint64_t> v;
        for (uint64_t i = 0; i < count; i++) {   // no up-front reserve: a lying count ends at EOF
            uint64_t b;
            if (!read_scalar(c, et, b, e)) return false;
            v.push_back(b);
        }
        nodes[idx].sc = std::move(v);
        return true;
    }
    if (et != STYX_GGUF_STRING && et != STYX_GGUF_ARRAY) {
        e = unknown_type(et);
        return false;
    }
    std::vector<uint64_t> kids;
    for (uint64_t i = 0; i < count; i++) {
        nodes.emplace_back();
        const size_t k = nodes.size() - 1;
        kids.push_back(k);
        if (!read_value(c, et, nodes, k, e, depth + 1)) return false;
    }
    nodes[idx].kids = std::move(kids);
    return true;
}

// compute_size_bytes (lib.rs:243-332): block elements and bytes per type
bool type_size(uint32_t t, uint64_t &elems, uint64_t &bytes) {
    struct T {
        uint32_t type, elems, bytes;
    };
    static const T table[] = {
        {0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {6, 32, 22},   {7, 32, 24},
        {8, 32, 34},   {9, 32, 36},   {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
        {14, 256, 210}, {15, 256, 292}, {16, 256, 66}, {17, 256, 74},  {18, 256, 98},  {19, 256, 50},
        {20, 32, 18},  {21, 256, 110}, {22, 256, 82}, {23, 256, 136}, {24, 1, 1},     {25, 1, 2},
        {26, 1, 4},    {27, 1, 8},    {28, 1, 8},    {29, 256, 56},  {30, 1, 2}};
    for (const T &x : table)
        if (x.type == t) {
            elems = x.elems;
            bytes = x.bytes;
            return true;
        }
    return false;
}

bool size_bytes(const std::vector<uint64_t> &dims, uint32_t t, uint64_t &out, Error &e) {
    uint64_t be, bb;
    if (!type_size(t, be, bb)) {
        char m[64];
        std::snprintf(m, sizeof m, "Unknown ggml_type: %u", t);
        e = {STYX_EDATA, m};
        return false;
    }
    uint64_t product = 1;
    for (uint64_t d : dims) product *= d;   // wrapping, as the reference's release build
    if (product % be != 0) {
        e = {STYX_EDATA, "First dimension not multiple of block size"};
        return false;
    }
    out = (product / be) * bb;
    return true;
}

}  // namespace

struct styx_gguf {
    uint32_t version = 0;
    uint64_t data_start = 0;
    const uint8_t *data = nullptr;   // the file (mapped) or the caller's buffer
    uint64_t bytes = 0;
    void *map = nullptr;             // non-null when this handle owns a mapping
    std::vector<Node> nodes;
    std::vector<std::pair<std::string, uint64_t>> kvs;   // key, value node
    std::unordered_map<std::string, uint64_t> kv_index;
    std::vector<Tensor> tensors;
};

namespace {

int parse(styx_gguf *g) {
    Cursor c{g->data, g->data, g->data + g->bytes};
    Error e{STYX_OK, ""};
    uint32_t magic, version;
    uint64_t n_tensors, n_kv;
    if (!c.get(magic, e)) return styx::set_error(e.code, e.msg.c_str());
    if (magic != kMagic) return styx::set_error(STYX_EDATA, "Invalid GGUF magic");
    if (!c.get(version, e)) return styx::set_error(e.code, e.msg.c_str());
    if (version != 2 && version != 3) return styx::set_error(STYX_EDATA, "Unsupported GGUF version");
    if (!c.get(n_tensors, e) || !c.get(n_kv, e)) return styx::set_error(e.code, e.msg.c_str());
    g->version = version;
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key;
        uint32_t vt;
        if (!read_string(c, key, e) || !c.get(vt, e)) return styx::set_error(e.code, e.msg.c_str());
        g->nodes.emplace_back();
        const uint64_t node = g->nodes.size() - 1;
        if (!read_value(c, vt, g->nodes, node, e)) return styx::set_error(e.code, e.msg.c_str());
        auto it = g->kv_index.find(key);
        if (it != g->kv_index.end()) {
            g->kvs[it->second].second = node;   // HashMap insert: the later value wins
        } else {
            g->kv_index.emplace(key, g->kvs.size());
            g->kvs.emplace_back(std::move(key), node);
        }
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
        Tensor t;
        uint32_t nd;
        if (!read_string(c, t.name, e) || !c.get(nd, e)) return styx::set_error(e.code, e.msg.c_str());
        for (uint32_t d = 0; d < nd; d++) {
            uint64_t v;
            if (!c.get(v, e)) return styx::set_error(e.code, e.msg.c_str());
            t.dims.push_back(v);
        }
        if (!c.get(t.type, e) || !c.get(t.offset, e)) return styx::set_error(e.code, e.msg.c_str());
        if (!size_bytes(t.dims, t.type, t.size, e)) return styx::set_error(e.code, e.msg.c_str());
        g->tensors.push_back(std::move(t));
    }
    // general.alignment when it is a u32, else 32; round-up of lib.rs:111
    uint64_t alignment = 32;
    auto it = g->kv_index.find("general.alignment");
    if (it != g->kv_index.end()) {
        const Node &n = g->nodes[g->kvs[it->second].second];
        if (n.type == STYX_GGUF_U32) alignment = n.bits;
    }
    const uint64_t pos = c.pos();
    g->data_start = (pos + alignment - 1) & ~(alignment - 1);
    return STYX_OK;
}

const Node *node_of(const styx_gguf *g, uint64_t node) {
    return (g && node < g->nodes.size()) ? &g->nodes[node] : nullptr;
}

int bad_arg(const char *m) { return styx::set_error(STYX_EINVAL, m); }

}  // namespace

extern "C" {

int styx_gguf_open(const char *path, styx_gguf **out) {
    if (!path || !out) return bad_arg("null pointer");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        const std::string m = std::string(path) + ": " + std::strerror(errno);
        return styx::set_error(STYX_EIO, m.c_str());
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        const std::string m = std::string(path) + ": " + std::strerror(errno);
        ::close(fd);
        return styx::set_error(STYX_EIO, m.c_str());
    }
    styx_gguf *g = new (std::nothrow) styx_gguf;
    if (!g) {
        ::close(fd);
        return styx::set_error(STYX_ENOMEM, "out of memory");
    }
    g->bytes = static_cast<uint64_t>(st.st_size);
    if (g->bytes) {
        void *m = mmap(nullptr, g->bytes, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) {
            const std::string msg = std::string(path) + ": mmap: " + std::strerror(errno);
            ::close(fd);
            delete g;
            return styx::set_error(STYX_EIO, msg.c_str());
        }
        g->map = m;
        g->data = static_cast<const uint8_t *>(m);
    }
    ::close(fd);   // the mapping stays valid
    int rc;
    try {
        rc = parse(g);
    } catch (const std::bad_alloc &) {
        rc = styx::set_error(STYX_ENOMEM, "out of memory while parsing");
    }
    if (rc != STYX_OK) {
        styx_gguf_close(g);
        return rc;
    }
    *out = g;
    return STYX_OK;
}

int styx_gguf_open_memory(const void *data, uint64_t bytes, styx_gguf **out) {
    if (!out || (!data && bytes)) return bad_arg("null pointer");
    *out = nullptr;
    styx_gguf *g = new (std::nothrow) styx_gguf;
    if (!g) return styx::set_error(STYX_ENOMEM, "out of memory");
    g->data = static_cast<const uint8_t *>(data);
    g->bytes = bytes;
    int rc;
    try {
        rc = parse(g);
    } catch (const std::bad_alloc &) {
        rc = styx::set_error(STYX_ENOMEM, "out of memory while parsing");
    }
    if (rc != STYX_OK) {
        delete g;
        return rc;
    }
    *out = g;
    return STYX_OK;
}

void styx_gguf_close(styx_gguf *g) {
    if (!g) return;
    if (g->map) munmap(g->map, g->bytes);
    delete g;
}

uint32_t styx_gguf_version(const styx_gguf *g) { return g ? g->version : 0; }
uint64_t styx_gguf_data_start(const styx_gguf *g) { return g ? g->data_start : 0; }
uint64_t styx_gguf_file_bytes(const styx_gguf *g) { return g ? g->bytes : 0; }

uint64_t styx_gguf_kv_count(const styx_gguf *g) { return g ? g->kvs.size() : 0; }

int styx_gguf_kv_key(const styx_gguf *g, uint64_t i, const char **key) {
    if (!g || !key) return bad_arg("null pointer");
    if (i >= g->kvs.size()) return bad_arg("key index out of range");
    *key = g->kvs[i].first.c_str();
    return STYX_OK;
}

int styx_gguf_kv_value(const styx_gguf *g, uint64_t i, uint64_t *node) {
    if (!g || !node) return bad_arg("null pointer");
    if (i >= g->kvs.size()) return bad_arg("key index out of range");
    *node = g->kvs[i].second;
    return STYX_OK;
}

int64_t styx_gguf_find_kv(const styx_gguf *g, const char *key) {
    if (!g || !key) return -1;
    auto it = g->kv_index.find(key);
    return it == g->kv_index.end() ? -1 : static_cast<int64_t>(it->second);
}

int styx_gguf_node_type(const styx_gguf *g, uint64_t node, uint32_t *vtype, uint32_t *elem_type, uint64_t *count) {
    const Node *n = node_of(g, node);
    if (!n) return bad_arg("no such node");
    if (vtype) *vtype = n->type;
    if (elem_type) *elem_type = n->elem;
    if (count) *count = n->count;
    return STYX_OK;
}

int styx_gguf_node_scalar(const styx_gguf *g, uint64_t node, uint64_t index, void *out) {
    const Node *n = node_of(g, node);
    if (!n || !out) return bad_arg("no such node / null pointer");
    uint64_t bits;
    uint32_t t;
    if (n->type == STYX_GGUF_ARRAY) {
        if (!scalar_bytes(n->elem)) return bad_arg("not an array of scalars");
        if (index >= n->sc.size()) return bad_arg("array index out of range");
        bits = n->sc[index];
        t = n->elem;
    } else {
        if (!scalar_bytes(n->type)) return bad_arg("not a scalar");
        if (index != 0) return bad_arg("index of a scalar must be 0");
        bits = n->bits;
        t = n->type;
    }
    std::memcpy(out, &bits, static_cast<size_t>(scalar_bytes(t)));
    return STYX_OK;
}

int styx_gguf_node_string(const styx_gguf *g, uint64_t node, uint64_t index, const char **s, uint64_t *len) {
    const Node *n = node_of(g, node);
    if (!n || !s || !len) return bad_arg("no such node / null pointer");
    if (n->type == STYX_GGUF_ARRAY) {
        if (n->elem != STYX_GGUF_STRING) return bad_arg("not an array of strings");
        if (index >= n->kids.size()) return bad_arg("array index out of range");
        n = &g->nodes[n->kids[index]];
    } else if (n->type != STYX_GGUF_STRING || index != 0) {
        return bad_arg("not a string");
    }
    *s = n->str.data();
    *len = n->str.size();
    return STYX_OK;
}

int styx_gguf_node_elem(const styx_gguf *g, uint64_t node, uint64_t index, uint64_t *elem) {
    const Node *n = node_of(g, node);
    if (!n || !elem) return bad_arg("no such node / null pointer");
    if (n->type != STYX_GGUF_ARRAY || n->elem != STYX_GGUF_ARRAY) return bad_arg("not an array of arrays");
    if (index >= n->kids.size()) return bad_arg("array index out of range");
    *elem = n->kids[index];
    return STYX_OK;
}

static const Node *typed(const styx_gguf *g, const char *key, uint32_t want) {
    const int64_t i = styx_gguf_find_kv(g, key);
    if (i < 0) return nullptr;
    const Node &n = g->nodes[g->kvs[static_cast<size_t>(i)].second];
    return n.type == want ? &n : nullptr;
}

int styx_gguf_get_u32(const styx_gguf *g, const char *key, uint32_t *out) {
    if (!g || !key || !out) return bad_arg("null pointer");
    const Node *n = typed(g, key, STYX_GGUF_U32);
    if (!n) return styx::set_error(STYX_EINVAL, (std::string("missing/unexpected ") + key).c_str());
    *out = static_cast<uint32_t>(n->bits);
    return STYX_OK;
}

int styx_gguf_get_f32(const styx_gguf *g, const char *key, float *out) {
    if (!g || !key || !out) return bad_arg("null pointer");
    const Node *n = typed(g, key, STYX_GGUF_F32);
    if (!n) return styx::set_error(STYX_EINVAL, (std::string("missing/unexpected ") + key).c_str());
    const uint32_t b = static_cast<uint32_t>(n->bits);
    std::memcpy(out, &b, 4);
    return STYX_OK;
}

int styx_gguf_get_str(const styx_gguf *g, const char *key, const char **s, uint64_t *len) {
    if (!g || !key || !s || !len) return bad_arg("null pointer");
    const Node *n = typed(g, key, STYX_GGUF_STRING);
    if (!n) return styx::set_error(STYX_EINVAL, (std::string("missing/unexpected ") + key).c_str());
    *s = n->str.data();
    *len = n->str.size();
    return STYX_OK;
}

uint64_t styx_gguf_tensor_count(const styx_gguf *g) { return g ? g->tensors.size() : 0; }

int styx_gguf_tensor(const styx_gguf *g, uint64_t i, styx_gguf_tensor_info *out) {
    if (!g || !out) return bad_arg("null pointer");
    if (i >= g->tensors.size()) return bad_arg("tensor index out of range");
    const Tensor &t = g->tensors[i];
    out->name = t.name.c_str();
    out->n_dims = static_cast<uint32_t>(t.dims.size());
    out->dims = t.dims.data();
    out->ggml_type = t.type;
    out->offset = t.offset;
    out->size_bytes = t.size;
    return STYX_OK;
}

int64_t styx_gguf_find_tensor(const styx_gguf *g, const char *name) {
    if (!g || !name) return -1;
    for (size_t i = 0; i < g->tensors.size(); i++)
        if (g->tensors[i].name == name) return static_cast<int64_t>(i);
    return -1;
}

int styx_gguf_tensor_data(const styx_gguf *g, uint64_t i, const void **data) {
    if (!g || !data) return bad_arg("null pointer");
    if (i >= g->tensors.size()) return bad_arg("tensor index out of range");
    const Tensor &t = g->tensors[i];
    const uint64_t a = g->data_start, b = t.offset, n = t.size;
    // [a + b, a + b + n) inside the file, without overflow
    if (a > g->bytes || b > g->bytes - a || n > g->bytes - a - b) {
        const std::string m = "tensor " + t.name + ": bytes [data_start + offset, + size) lie outside the file";
        return styx::set_error(STYX_EDATA, m.c_str());
    }
    *data = g->data + a + b;
    return STYX_OK;
}

int styx_gguf_type_size(uint32_t ggml_type, uint64_t *block_elems, uint64_t *block_bytes) {
    if (!block_elems || !block_bytes) return bad_arg("null pointer");
    if (!type_size(ggml_type, *block_elems, *block_bytes)) {
        char m[64];
        std::snprintf(m, sizeof m, "Unknown ggml_type: %u", ggml_type);
        return styx::set_error(STYX_EDATA, m);
    }
    return STYX_OK;
}

int styx_gguf_tensor_bytes(uint32_t ggml_type, const uint64_t *dims, uint32_t n_dims, uint64_t *out) {
    if (!out || (!dims && n_dims)) return bad_arg("null pointer");
    Error e{STYX_OK, ""};
    std::vector<uint64_t> d(dims, dims + n_dims);
    if (!size_bytes(d, ggml_type, *out, e)) return styx::set_error(e.code, e.msg.c_str());
    return STYX_OK;
}

}  // extern "C"
