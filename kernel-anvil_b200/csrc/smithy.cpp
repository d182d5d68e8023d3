// smithy.cpp -- runtime {nwarps, rows_per_block} table for the MMVQ launcher.
//
// Behavioural replacement for the reference's header-only loader
// (patches/smithy-config.h:30-331), exported through the C ABI in include/anvil.h:
//   - table [41 ggml types][5 N buckets][5 K buckets], {0,0} = no override (:52);
//   - buckets <=128 / <=1024 / <=4096 / <=16384 / larger (:44-50);
//   - lazy load at first lookup, first success wins: $SMITHY_CONFIG, then
//     $HOME/.cache/smithy/<model stem>.json (stem from set_model or $SMITHY_MODEL), then
//     $HOME/.cache/smithy/default.json (:268-317);
//   - files larger than 1 MiB or empty are refused (:96); a cell is accepted only when
//     both values are in 1..32 (:246); the table counts as loaded when at least one cell
//     was accepted, and one line is logged to stderr (:259-265);
//   - readers take a shared lock, set_model / load take an exclusive one (:56-66).
// The JSON walk keeps the reference's scanning rules (so existing configs load to the same
// table, malformed ones included): inside the "configs" object every string token that
// starts with a digit and is followed by `: {` names a type; inside a type object every
// string token that scans as "<int>,<int>" with both in 0..4 and is followed by `: {`
// names a cell; a cell takes the integer after the first "nwarps" and "rows_per_block"
// keys within it.  Braces inside strings do not count toward nesting.
#include <atomic>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <vector>

#include "anvil.h"

namespace {

constexpr int kTypes = 41;  // GGML_TYPE_COUNT (kernel_anvil/codegen.py:32)
constexpr int kBuckets = 5;
constexpr long kMaxFileBytes = 1024 * 1024;

struct Cell {
    int nwarps;
    int rows_per_block;
};

Cell g_table[kTypes][kBuckets][kBuckets];
std::atomic<bool> g_loaded{false};
std::atomic<bool> g_attempted{false};
char g_model_path[512];
std::shared_mutex g_mu;

int bucket_of(int dim) {
    if (dim <= 128) return 0;
    if (dim <= 1024) return 1;
    if (dim <= 4096) return 2;
    if (dim <= 16384) return 3;
    return 4;
}

// Character-level helpers over [begin, end) of a NUL-terminated buffer.  Searches stop at
// `end` or at an embedded NUL, whichever comes first.
class JsonText {
  public:
    JsonText(const char *begin, const char *end) : begin_(begin), end_(end) {}

    const char *find(const char *from, char ch, const char *limit) const {
        for (const char *c = from; c < limit && *c; ++c)
            if (*c == ch) return c;
        return nullptr;
    }

    static const char *skip_space(const char *c, const char *limit) {
        while (c < limit && (*c == ' ' || *c == '\t' || *c == '\n' || *c == '\r')) ++c;
        return c;
    }

    // `open` points at a '"'; returns the position just past the closing quote
    // (backslash escapes honoured) or `limit` when unterminated.
    static const char *past_string(const char *open, const char *limit) {
        const char *c = open + 1;
        while (c < limit && *c != '"') c += (*c == '\\' && c + 1 < limit) ? 2 : 1;
        return c < limit ? c + 1 : c;
    }

    // `open` points at '{'; returns its matching '}' or nullptr.
    static const char *closing_brace(const char *open, const char *limit) {
        if (!open || *open != '{') return nullptr;
        int depth = 0;
        for (const char *c = open; c < limit;) {
            if (*c == '"') {
                c = past_string(c, limit);
                continue;
            }
            if (*c == '{') ++depth;
            if (*c == '}' && --depth == 0) return c;
            ++c;
        }
        return nullptr;
    }

    // `quote` points at (or just before) the closing quote of a key; returns the '{' of
    // the key's value when that value is an object, else nullptr.
    static const char *object_value(const char *quote, const char *limit) {
        if (!quote || quote >= limit) return nullptr;
        const char *c = quote;
        if (*c == '"') ++c;
        c = skip_space(c, limit);
        if (c >= limit || *c != ':') return nullptr;
        c = skip_space(c + 1, limit);
        return (c < limit && *c == '{') ? c : nullptr;
    }

    const char *begin() const { return begin_; }
    const char *end() const { return end_; }

  private:
    const char *begin_;
    const char *end_;
};

// Reads {nwarps, rows_per_block} out of one cell object [open, close].
bool read_cell(const char *open, const char *close, Cell *out) {
    const char *nw_key = strstr(open, "\"nwarps\"");
    const char *rpb_key = strstr(open, "\"rows_per_block\"");
    if (!nw_key || nw_key >= close || !rpb_key || rpb_key >= close) return false;
    const char *nw_colon = strchr(nw_key + 8, ':');
    const char *rpb_colon = strchr(rpb_key + 16, ':');
    const int nw = (nw_colon && nw_colon < close) ? atoi(nw_colon + 1) : 0;
    const int rpb = (rpb_colon && rpb_colon < close) ? atoi(rpb_colon + 1) : 0;
    if (nw < 1 || nw > 32 || rpb < 1 || rpb > 32) return false;
    out->nwarps = nw;
    out->rows_per_block = rpb;
    return true;
}

// Walks the cells of one type object (open, close) into the table; returns cells taken,
// or -1 when the walk had to stop (unbalanced cell object).
int read_type(const JsonText &t, int type, const char *open, const char *close) {
    int taken = 0;
    const char *c = open;
    while (c < close) {
        const char *q = t.find(c, '"', close);
        if (!q) break;
        const char *key = q + 1;
        int nb = -1, kb = -1;
        if (sscanf(key, "%d,%d", &nb, &kb) == 2 && nb >= 0 && nb < kBuckets && kb >= 0 &&
            kb < kBuckets) {
            const char *key_end = t.find(key, '"', close);
            if (!key_end) break;
            const char *cell_open = JsonText::object_value(key_end, close);
            if (!cell_open) {
                c = key_end + 1;
                continue;
            }
            const char *cell_close = JsonText::closing_brace(cell_open, close);
            if (!cell_close) break;
            Cell v;
            if (read_cell(cell_open, cell_close, &v)) {
                g_table[type][nb][kb] = v;
                ++taken;
            }
            c = cell_close + 1;
            continue;
        }
        c = key + 1;  // resume one past the character after the quote
    }
    return taken;
}

// Parses a whole document into the table.  Returns the number of cells accepted, or -1
// when there is no "configs" object at all.
int parse_document(const char *buf, size_t size) {
    const char *anchor = strstr(buf, "\"configs\"");
    if (!anchor) return -1;
    const JsonText t(buf, buf + size);
    const char *cfg_open = JsonText::object_value(anchor + strlen("\"configs\""), t.end());
    if (!cfg_open) return -1;
    const char *cfg_close = JsonText::closing_brace(cfg_open, t.end());
    if (!cfg_close) return -1;
    int taken = 0;
    const char *c = cfg_open;
    while (c && c < cfg_close) {
        const char *q = t.find(c, '"', cfg_close);
        if (!q) break;
        const char *key = q + 1;
        if (!isdigit(static_cast<unsigned char>(*key))) {
            c = key;
            continue;
        }
        const int type = atoi(key);
        const char *key_end = t.find(key, '"', cfg_close);
        if (!key_end) break;
        const char *type_open = JsonText::object_value(key_end, cfg_close);
        if (!type_open) {
            c = key_end + 1;
            continue;
        }
        if (type < 0 || type >= kTypes) {
            c = type_open;  // keep scanning from inside the skipped object
            continue;
        }
        const char *type_close = JsonText::closing_brace(type_open, cfg_close);
        if (!type_close) break;
        taken += read_type(t, type, type_open, type_close);
        c = type_close + 1;
    }
    return taken;
}

// Loads one file into the table (caller holds the exclusive lock).  Returns cells
// accepted (>= 0) or a negative status when the file is unreadable, empty, over 1 MiB,
// or has no "configs" object; the loaded flag is only updated after a full parse.
int load_locked(const char *path) {
    if (!path) return ANVIL_ERR_INVALID;
    FILE *f = fopen(path, "r");
    if (!f) return ANVIL_ERR_INVALID;
    fseek(f, 0, SEEK_END);
    const long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (size <= 0 || size > kMaxFileBytes) {
        fclose(f);
        return ANVIL_ERR_INVALID;
    }
    std::vector<char> buf(size_t(size) + 1, '\0');
    const size_t got = fread(buf.data(), 1, size_t(size), f);
    fclose(f);
    buf[got] = '\0';
    const int taken = parse_document(buf.data(), size_t(size));
    if (taken < 0) return ANVIL_ERR_INVALID;
    g_loaded.store(taken > 0, std::memory_order_release);
    if (taken > 0) fprintf(stderr, "kernel-anvil: loaded %d shape configs from %s\n", taken, path);
    return taken;
}

void try_load_locked() {
    const char *env_cfg = getenv("SMITHY_CONFIG");
    if (env_cfg && load_locked(env_cfg) > 0) return;
    const char *home = getenv("HOME");
    if (!home) return;
    const char *model = g_model_path;
    const char *env_model = getenv("SMITHY_MODEL");
    if (model[0] == '\0' && env_model) model = env_model;
    if (model[0] != '\0') {
        const char *slash = strrchr(model, '/');
        if (!slash) slash = strrchr(model, '\\');
        const char *base = slash ? slash + 1 : model;
        size_t len = strlen(base);
        const char *dot = strrchr(base, '.');
        if (dot && dot > base) len = size_t(dot - base);
        std::string stem(base, len < 255 ? len : 255);
        char path[512];
        snprintf(path, sizeof(path), "%s/.cache/smithy/%s.json", home, stem.c_str());
        if (load_locked(path) > 0) return;
    }
    char path[512];
    snprintf(path, sizeof(path), "%s/.cache/smithy/default.json", home);
    load_locked(path);
}

}  // namespace

extern "C" {

int anvil_smithy_bucket(int dim) { return bucket_of(dim); }

void anvil_smithy_set_model(const char *path) {
    if (!path) return;
    std::unique_lock<std::shared_mutex> lk(g_mu);
    size_t len = strlen(path);
    if (len >= sizeof(g_model_path)) len = sizeof(g_model_path) - 1;
    memcpy(g_model_path, path, len);
    g_model_path[len] = '\0';
    // Flags first, then the table: a reader that saw loaded == true never pairs it with
    // a half-cleared table.
    g_loaded.store(false, std::memory_order_release);
    g_attempted.store(false, std::memory_order_release);
    memset(g_table, 0, sizeof(g_table));
}

int anvil_smithy_load(const char *path) {
    std::unique_lock<std::shared_mutex> lk(g_mu);
    return load_locked(path);
}

int anvil_smithy_try_load(void) {
    if (g_loaded.load(std::memory_order_acquire)) return 1;
    if (g_attempted.load(std::memory_order_acquire)) return 0;
    std::unique_lock<std::shared_mutex> lk(g_mu);
    if (g_loaded.load(std::memory_order_relaxed)) return 1;
    if (g_attempted.load(std::memory_order_relaxed)) return 0;
    g_attempted.store(true, std::memory_order_release);
    try_load_locked();
    return g_loaded.load(std::memory_order_relaxed) ? 1 : 0;
}

int anvil_smithy_lookup(int ggml_type, int nrows, int ncols, int *nwarps, int *rows_per_block) {
    anvil_smithy_try_load();
    std::shared_lock<std::shared_mutex> lk(g_mu);
    Cell v = {0, 0};
    if (g_loaded.load(std::memory_order_acquire) && ggml_type >= 0 && ggml_type < kTypes)
        v = g_table[ggml_type][bucket_of(nrows)][bucket_of(ncols)];
    if (nwarps) *nwarps = v.nwarps;
    if (rows_per_block) *rows_per_block = v.rows_per_block;
    return (v.nwarps > 0 || v.rows_per_block > 0) ? 1 : 0;
}

void anvil_smithy_reset(void) {
    std::unique_lock<std::shared_mutex> lk(g_mu);
    g_model_path[0] = '\0';
    g_loaded.store(false, std::memory_order_release);
    g_attempted.store(false, std::memory_order_release);
    memset(g_table, 0, sizeof(g_table));
}

}  // extern "C"
