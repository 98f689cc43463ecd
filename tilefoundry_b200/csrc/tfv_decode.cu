// Native decode of schedule documents into the packed layout of the C ABI.
//
// Host code only. tfv_decode_schedules parses strict schedule JSON documents
// (serialization.py:679-727 and the JSON rules of serialization.py:59-142: duplicate
// fields, non-finite numbers and NaN/Infinity constants rejected, exact field sets,
// integers that are JSON integers and not booleans), applies the schedule record
// constructors (model.py:425-507), and writes each accepted document as dense timing
// rows plus a frame index into a tfv_frameset, which deduplicates lanes + sync sets
// exactly like the Python packer (FrameSet.add / pack_rows). Documents are decoded on
// several host threads; frames are numbered in document order.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "tfv.h"

int tfv_internal_fail(int code, const char* message);

namespace {

using i128 = __int128;
constexpr i128 kIntCap = static_cast<i128>(1) << 120;  // parsed integers saturate here

// ---------------------------------------------------------------------------------------
// JSON values (a small DOM per document)
// ---------------------------------------------------------------------------------------

struct Value {
    enum Kind : uint8_t { Null, Bool, Int, Float, Str, Arr, Obj } kind = Null;
    bool ascii = true;  // strings: every code point below 128
    i128 num = 0;
    std::string str;
    std::vector<Value> items;                         // arrays
    std::vector<std::pair<std::string, Value>> keys;  // objects (insertion order)
};

class Parser {
  public:
    Parser(const char* s, size_t n) : p_(s), end_(s + n) {}

    bool parse(Value& out) {
        ws();
        if (!value(out, 0)) return false;
        ws();
        return p_ == end_;  // "Extra data" otherwise
    }

  private:
    const char* p_;
    const char* end_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* word) {
        const size_t n = std::strlen(word);
        if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, word, n) != 0) return false;
        p_ += n;
        return true;
    }

    bool value(Value& v, int depth) {
        if (depth > 256 || p_ >= end_) return false;
        const char c = *p_;
        if (c == '{') return object(v, depth);
        if (c == '[') return array(v, depth);
        if (c == '"') {
            v.kind = Value::Str;
            return string(v.str, v.ascii);
        }
        if (c == 't') {
            v.kind = Value::Bool;
            return lit("true");
        }
        if (c == 'f') {
            v.kind = Value::Bool;
            return lit("false");
        }
        if (c == 'n') {
            v.kind = Value::Null;
            return lit("null");
        }
        if (c == '-' || (c >= '0' && c <= '9')) return number(v);
        return false;  // NaN / Infinity constants and everything else
    }

    bool number(Value& v) {
        bool neg = false;
        if (*p_ == '-') {
            neg = true;
            ++p_;
        }
        if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
        i128 mag = 0;
        if (*p_ == '0') {
            ++p_;
        } else {
            int digits = 0;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') {
                mag = mag * 10 + (*p_ - '0');
                if (mag > kIntCap) mag = kIntCap;
                ++p_;
                ++digits;
            }
            if (digits > 4300) return false;  // Python's int() refuses longer decimal strings
        }
        bool is_float = false;
        if (p_ < end_ && *p_ == '.') {
            ++p_;
            if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
            is_float = true;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
            is_float = true;
        }
        // A float is never an accepted field value here, so its finiteness does not matter.
        v.kind = is_float ? Value::Float : Value::Int;
        v.num = neg ? -mag : mag;
        return true;
    }

    static int hex(char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }

    bool u4(unsigned& cp) {
        if (end_ - p_ < 4) return false;
        cp = 0;
        for (int i = 0; i < 4; ++i) {
            const int h = hex(p_[i]);
            if (h < 0) return false;
            cp = cp * 16 + static_cast<unsigned>(h);
        }
        p_ += 4;
        return true;
    }

    // Decodes a string; code points >= 128 are kept only as a non-ASCII mark (no
    // identifier, field name or format string the schema accepts contains one).
    bool string(std::string& out, bool& ascii) {
        ++p_;  // opening quote
        out.clear();
        ascii = true;
        while (p_ < end_) {
            const unsigned char c = static_cast<unsigned char>(*p_);
            if (c == '"') {
                ++p_;
                return true;
            }
            if (c < 0x20) return false;  // control characters are invalid in strict JSON
            if (c == '\\') {
                ++p_;
                if (p_ >= end_) return false;
                const char e = *p_++;
                switch (e) {
                    case '"': out.push_back('"'); break;
                    case '\\': out.push_back('\\'); break;
                    case '/': out.push_back('/'); break;
                    case 'b': out.push_back('\b'); break;
                    case 'f': out.push_back('\f'); break;
                    case 'n': out.push_back('\n'); break;
                    case 'r': out.push_back('\r'); break;
                    case 't': out.push_back('\t'); break;
                    case 'u': {
                        unsigned cp;
                        if (!u4(cp)) return false;
                        if (cp < 0x80) {
                            out.push_back(static_cast<char>(cp));
                        } else {
                            ascii = false;
                            out.push_back('\x7f');  // placeholder: never part of an accepted name
                            // a high surrogate followed by an escaped low surrogate is one code point
                            if (cp >= 0xD800 && cp <= 0xDBFF && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                                const char* save = p_;
                                p_ += 2;
                                unsigned lo;
                                if (!u4(lo) || lo < 0xDC00 || lo > 0xDFFF) p_ = save;
                            }
                        }
                        break;
                    }
                    default: return false;
                }
                continue;
            }
            if (c >= 0x80) {
                ascii = false;
                out.push_back('\x7f');
                ++p_;
                while (p_ < end_ && (static_cast<unsigned char>(*p_) & 0xC0) == 0x80) ++p_;  // UTF-8 continuation
                continue;
            }
            out.push_back(static_cast<char>(c));
            ++p_;
        }
        return false;
    }

    bool array(Value& v, int depth) {
        v.kind = Value::Arr;
        ++p_;
        ws();
        if (p_ < end_ && *p_ == ']') {
            ++p_;
            return true;
        }
        while (true) {
            v.items.emplace_back();
            ws();
            if (!value(v.items.back(), depth + 1)) return false;
            ws();
            if (p_ >= end_) return false;
            if (*p_ == ',') {
                ++p_;
                continue;
            }
            if (*p_ == ']') {
                ++p_;
                return true;
            }
            return false;
        }
    }

    bool object(Value& v, int depth) {
        v.kind = Value::Obj;
        ++p_;
        ws();
        if (p_ < end_ && *p_ == '}') {
            ++p_;
            return true;
        }
        while (true) {
            ws();
            if (p_ >= end_ || *p_ != '"') return false;
            std::string key;
            bool key_ascii;
            if (!string(key, key_ascii)) return false;
            if (!key_ascii) key.push_back('\x7f');
            ws();
            if (p_ >= end_ || *p_ != ':') return false;
            ++p_;
            ws();
            Value item;
            if (!value(item, depth + 1)) return false;
            for (const auto& kv : v.keys)
                if (kv.first == key) return false;  // duplicate JSON field
            v.keys.emplace_back(std::move(key), std::move(item));
            ws();
            if (p_ >= end_) return false;
            if (*p_ == ',') {
                ++p_;
                continue;
            }
            if (*p_ == '}') {
                ++p_;
                return true;
            }
            return false;
        }
    }
};

// ---------------------------------------------------------------------------------------
// Schema and record rules
// ---------------------------------------------------------------------------------------

// [A-Za-z_][A-Za-z0-9_.-]* in ASCII (the identifier rule of the records).
bool is_identifier(const Value& v) {
    if (v.kind != Value::Str || !v.ascii || v.str.empty()) return false;
    const char c0 = v.str[0];
    if (!((c0 >= 'A' && c0 <= 'Z') || (c0 >= 'a' && c0 <= 'z') || c0 == '_')) return false;
    for (char c : v.str)
        if (!((c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') || c == '_' || c == '.' ||
              c == '-'))
            return false;
    return true;
}

// The object's fields, exactly `names` (no unknown, none missing), in `names` order.
bool fields(const Value& v, std::initializer_list<const char*> names, const Value** out) {
    if (v.kind != Value::Obj || v.keys.size() != names.size()) return false;
    int i = 0;
    for (const char* name : names) {
        const Value* found = nullptr;
        for (const auto& kv : v.keys)
            if (kv.first == name) found = &kv.second;
        if (!found) return false;
        out[i++] = found;
    }
    return true;
}

struct Row {
    i128 iteration, start, issue_end, completion;
    std::string op;
};

struct Edge {
    std::string after, before;
    i128 distance;
    bool operator<(const Edge& o) const {
        if (after != o.after) return after < o.after;
        if (before != o.before) return before < o.before;
        return distance < o.distance;
    }
    bool operator==(const Edge& o) const { return after == o.after && before == o.before && distance == o.distance; }
};

struct Doc {
    std::vector<std::vector<std::string>> lanes;
    std::vector<Edge> sync;  // sorted
    std::vector<Row> rows;
};

// Decodes one document; false when the reference would raise WarpgroupSerializationError.
bool decode(const char* text, size_t n, Doc& d) {
    Value root;
    if (!Parser(text, n).parse(root)) return false;
    const Value* f[4];
    if (!fields(root, {"format", "lanes", "sync", "times"}, f)) return false;
    if (f[0]->kind != Value::Str || !f[0]->ascii || f[0]->str != TFV_SCHEDULE_FORMAT) return false;
    if (f[1]->kind != Value::Arr || f[2]->kind != Value::Arr || f[3]->kind != Value::Arr) return false;
    // lanes (WarpgroupLane, model.py:425-439)
    for (const Value& lane : f[1]->items) {
        if (lane.kind != Value::Arr) return false;
        d.lanes.emplace_back();
        for (const Value& op : lane.items) {
            if (!is_identifier(op)) return false;
            d.lanes.back().push_back(op.str);
        }
        std::vector<std::string> sorted = d.lanes.back();
        std::sort(sorted.begin(), sorted.end());
        if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end()) return false;
    }
    // sync edges (SynchronizationEdge, model.py:442-455)
    for (const Value& e : f[2]->items) {
        const Value* g[3];
        if (!fields(e, {"after", "before", "distance"}, g)) return false;
        if (!is_identifier(*g[0]) || !is_identifier(*g[1]) || g[2]->kind != Value::Int || g[2]->num < 0) return false;
        if (g[0]->str == g[1]->str && g[2]->num == 0) return false;
        d.sync.push_back(Edge{g[0]->str, g[1]->str, g[2]->num});
    }
    // timed instances (TimedOperation, model.py:458-477)
    for (const Value& r : f[3]->items) {
        if (r.kind != Value::Arr || r.items.size() != 5) return false;
        const Value* x = r.items.data();
        if (x[0].kind != Value::Int || !is_identifier(x[1]) || x[2].kind != Value::Int || x[3].kind != Value::Int ||
            x[4].kind != Value::Int)
            return false;
        const i128 it = x[0].num, s = x[2].num, e = x[3].num, c = x[4].num;
        if (it < 0 || s < 0 || e <= 0 || c <= 0 || e <= s || c < e) return false;
        d.rows.push_back(Row{it, s, e, c, x[1].str});
    }
    // the schedule (WarpgroupSchedule, model.py:480-507)
    if (d.lanes.empty()) return false;
    std::vector<std::string> all;
    for (const auto& lane : d.lanes) all.insert(all.end(), lane.begin(), lane.end());
    std::sort(all.begin(), all.end());
    if (std::adjacent_find(all.begin(), all.end()) != all.end()) return false;
    std::sort(d.sync.begin(), d.sync.end());
    if (std::adjacent_find(d.sync.begin(), d.sync.end()) != d.sync.end()) return false;
    std::vector<std::pair<i128, std::string>> inst;
    inst.reserve(d.rows.size());
    for (const Row& r : d.rows) inst.emplace_back(r.iteration, r.op);
    std::sort(inst.begin(), inst.end());
    if (std::adjacent_find(inst.begin(), inst.end()) != inst.end()) return false;
    return true;
}

std::string decimal(i128 v) {
    if (v == 0) return "0";
    const bool neg = v < 0;
    std::string out;
    while (v != 0) {
        const int digit = static_cast<int>(v % 10);
        out.push_back(static_cast<char>('0' + (digit < 0 ? -digit : digit)));
        v /= 10;
    }
    if (neg) out.push_back('-');
    std::reverse(out.begin(), out.end());
    return out;
}

int32_t clamp32(i128 v) {
    if (v > INT32_MAX) return INT32_MAX;
    if (v < INT32_MIN) return INT32_MIN;
    return static_cast<int32_t>(v);
}

}  // namespace

// ---------------------------------------------------------------------------------------
// Frame set: deduplicated lanes + sync sets in the layout of tfv_frames
// ---------------------------------------------------------------------------------------

struct tfv_frameset {
    int n_ops = 0;
    int iterations = 0;
    std::vector<std::string> op_ids;
    std::unordered_map<std::string, int> index;
    std::unordered_map<std::string, int> frame_of;  // canonical frame key -> frame
    std::unordered_map<std::string, int> set_of;    // canonical sorted sync key -> set
    std::vector<uint16_t> lane_pos;                 // [F][N]
    std::vector<int32_t> lane_count, flags, sync_set;
    std::vector<int32_t> sync_offsets{0};
    std::vector<int32_t> sync_edges;  // [E][3]

    int add(const Doc& d) {
        std::string set_key;
        for (const Edge& e : d.sync) {
            set_key += e.after;
            set_key += '\x01';
            set_key += e.before;
            set_key += '\x01';
            set_key += decimal(e.distance);
            set_key += '\x02';
        }
        std::string key;
        for (const auto& lane : d.lanes) {
            for (const auto& op : lane) {
                key += op;
                key += '\x01';
            }
            key += '\x02';
        }
        key += '\x03';
        key += set_key;
        auto found = frame_of.find(key);
        if (found != frame_of.end()) return found->second;
        int set_id;
        auto s = set_of.find(set_key);
        if (s != set_of.end()) {
            set_id = s->second;
        } else {
            set_id = static_cast<int>(sync_offsets.size()) - 1;
            set_of.emplace(set_key, set_id);
            for (const Edge& e : d.sync) {
                const auto a = index.find(e.after), b = index.find(e.before);
                sync_edges.push_back(a == index.end() ? -1 : a->second);
                sync_edges.push_back(b == index.end() ? -1 : b->second);
                sync_edges.push_back(static_cast<int32_t>(std::min<i128>(e.distance, TFV_TIME_LIMIT)));
            }
            sync_offsets.push_back(static_cast<int32_t>(sync_edges.size() / 3));
        }
        int fl = 0;
        std::vector<uint16_t> pos(n_ops, static_cast<uint16_t>(TFV_LANE_ABSENT << TFV_LANE_SHIFT));
        for (size_t l = 0; l < d.lanes.size(); ++l) {
            int position = 0;
            for (const auto& op : d.lanes[l]) {
                const auto k = index.find(op);
                if (k == index.end()) {
                    fl |= TFV_FRAME_UNKNOWN_LANE_OP;
                    continue;
                }
                if (static_cast<int>(l) < TFV_MAX_LANES) {
                    pos[k->second] = static_cast<uint16_t>((static_cast<int>(l) << TFV_LANE_SHIFT) | position);
                    ++position;
                }
            }
        }
        const int id = static_cast<int>(lane_count.size());
        frame_of.emplace(std::move(key), id);
        lane_pos.insert(lane_pos.end(), pos.begin(), pos.end());
        lane_count.push_back(static_cast<int32_t>(d.lanes.size()));
        flags.push_back(fl);
        sync_set.push_back(set_id);
        return id;
    }
};

namespace {

// Rows of one decoded document in the dense [I][N] grid (pack_rows in batch.py).
void pack(const tfv_frameset& fs, const Doc& d, int32_t* start, int32_t* issue_end, int32_t* completion, int32_t& flags,
          int32_t& makespan, int32_t& ii) {
    const int N = fs.n_ops, I = fs.iterations;
    std::vector<uint8_t> present(static_cast<size_t>(N) * I, 0);
    flags = 0;
    for (const Row& r : d.rows) {
        const auto k = fs.index.find(r.op);
        if (k == fs.index.end() || r.iteration >= I) {
            flags |= TFV_ROWS_COVERAGE;
            continue;
        }
        i128 s = r.start, e = r.issue_end, c = r.completion;
        if (std::max(s, std::max(e, c)) >= TFV_TIME_LIMIT) {  // keeps the verdict "out of range"
            s = TFV_TIME_LIMIT;
            e = c = TFV_TIME_LIMIT + 1;
        }
        const size_t at = static_cast<size_t>(r.iteration) * N + k->second;
        start[at] = clamp32(s);
        issue_end[at] = clamp32(e);
        completion[at] = clamp32(c);
        present[at] = 1;
    }
    size_t first = present.size();
    for (size_t at = 0; at < present.size(); ++at)
        if (present[at]) {
            first = at;
            break;
        }
    bool missing = false;
    for (size_t at = 0; at < present.size(); ++at)
        if (!present[at]) missing = true;
    if (missing) {
        flags |= TFV_ROWS_COVERAGE;
        if (first < present.size())  // missing instances repeat a listed row
            for (size_t at = 0; at < present.size(); ++at)
                if (!present[at]) {
                    start[at] = start[first];
                    issue_end[at] = issue_end[first];
                    completion[at] = completion[first];
                }
    }
    makespan = ii = 0;
    if (flags) {  // makespan and II over the rows as listed (verify.py:261-262, api.py:29-33)
        i128 mk = 0;
        const Row *s1 = nullptr, *s2 = nullptr;
        for (const Row& r : d.rows) {
            mk = std::max(mk, r.completion);
            if (N > 0 && r.op == fs.op_ids[0]) {
                if (r.iteration == 1) s1 = &r;
                if (r.iteration == 2) s2 = &r;
            }
        }
        makespan = clamp32(mk);
        if (I >= 3 && s1 && s2) ii = clamp32(s2->start - s1->start);
    }
}

}  // namespace

extern "C" {

int tfv_frameset_create(int n_ops, int iterations, const char* const* op_ids, tfv_frameset** out) {
    if (!out || n_ops < 0 || iterations < 1 || (n_ops > 0 && !op_ids))
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "need n_ops >= 0, iterations >= 1, op_ids and out");
    auto* fs = new tfv_frameset();
    fs->n_ops = n_ops;
    fs->iterations = iterations;
    for (int k = 0; k < n_ops; ++k) {
        if (!op_ids[k]) {
            delete fs;
            return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "op id is NULL");
        }
        fs->op_ids.emplace_back(op_ids[k]);
        if (k > 0 && !(fs->op_ids[k - 1] < fs->op_ids[k])) {
            delete fs;
            return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "op ids must be strictly increasing");
        }
        fs->index.emplace(fs->op_ids[k], k);
    }
    *out = fs;
    return TFV_OK;
}

int tfv_frameset_destroy(tfv_frameset* fs) {
    delete fs;
    return TFV_OK;
}

int tfv_frameset_view(const tfv_frameset* fs, tfv_frames* out) {
    if (!fs || !out) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "frameset and out must not be NULL");
    static const int32_t kNoEdge[3] = {0, 0, 0};
    out->n_frames = static_cast<int>(fs->lane_count.size());
    out->lane_pos = fs->lane_pos.data();
    out->lane_count = fs->lane_count.data();
    out->flags = fs->flags.data();
    out->sync_set = fs->sync_set.data();
    out->n_sync_sets = static_cast<int>(fs->sync_offsets.size()) - 1;
    out->n_sync_edges = static_cast<int>(fs->sync_edges.size() / 3);
    out->sync_offsets = fs->sync_offsets.data();
    out->sync_edges = fs->sync_edges.empty() ? kNoEdge : fs->sync_edges.data();
    return TFV_OK;
}

int tfv_decode_schedules(tfv_frameset* fs, int64_t n, const char* const* documents, const size_t* lengths,
                         int32_t* start, int32_t* issue_end, int32_t* completion, int32_t* frame, int32_t* row_flags,
                         int32_t* makespan_override, int32_t* ii_override, int32_t* status, int threads) {
    if (!fs || n < 0) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "frameset is NULL or n < 0");
    if (n == 0) return TFV_OK;
    if (!documents || !lengths || !start || !issue_end || !completion || !frame || !row_flags || !makespan_override ||
        !ii_override || !status)
        return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "array arguments must not be NULL");
    const size_t cell = static_cast<size_t>(fs->n_ops) * fs->iterations;
    std::vector<Doc> docs(static_cast<size_t>(n));
    std::atomic<int64_t> next{0};
    auto work = [&]() {
        for (int64_t c; (c = next.fetch_add(1)) < n;) {
            int32_t* s = start + c * cell;
            int32_t* e = issue_end + c * cell;
            int32_t* cp = completion + c * cell;
            std::fill(s, s + cell, 0);
            std::fill(e, e + cell, 1);
            std::fill(cp, cp + cell, 1);
            row_flags[c] = makespan_override[c] = ii_override[c] = 0;
            const bool ok = documents[c] && decode(documents[c], lengths[c], docs[c]);
            status[c] = ok ? 0 : 1;
            if (ok) pack(*fs, docs[c], s, e, cp, row_flags[c], makespan_override[c], ii_override[c]);
        }
    };
    int t = threads > 0 ? threads : static_cast<int>(std::thread::hardware_concurrency());
    t = std::max(1, std::min<int>(t, static_cast<int>(std::min<int64_t>(n, 64))));
    std::vector<std::thread> pool;
    for (int i = 1; i < t; ++i) pool.emplace_back(work);
    work();
    for (auto& th : pool) th.join();
    for (int64_t c = 0; c < n; ++c) frame[c] = status[c] == 0 ? fs->add(docs[c]) : -1;
    return TFV_OK;
}

}  // extern "C"
