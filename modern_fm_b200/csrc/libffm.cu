// libffm.cu — libffm text reader (host, native, multi-threaded).
//
// The reference reads libffm files in pure Python (load_libffm,
// python/modern_fm/libffm.py:31-83): one example per line,
// `<label> <field>:<feature>:<value> ...`, builds a scipy CSR through COO
// (which sums duplicate entries), a float64 label vector and an int64 field id
// per feature. mfm_libffm_read is its reader half: the file is cut into
// chunks at line boundaries, each chunk parsed by its own thread, and the
// per-chunk rows concatenated in file order into a raw CSR in the boundary
// format (entries in file order, duplicates kept); mfm_csr_prep_device then
// canonicalises that CSR on the GPU (sorting, duplicate sums, narrowing).
//
// Parsing follows the reference token for token: lines split as Python's
// universal newlines do (\n, \r\n, \r), blank lines skipped but counted,
// tokens split on whitespace, the label read by float(), every other token
// split on ':' into exactly three parts read by int(), int(), float()
// (optional sign, digits with single underscores between digits; floats also
// take a fraction, an exponent and inf / infinity / nan in any case). Values
// are rounded correctly, as Python's float() rounds them (Clinger's exact
// fast path where it applies, strtod in the "C" locale otherwise), so every
// value is bitwise the reference's. Errors carry the reference's
// messages and line numbers, and the first error in file order wins (a
// feature's field conflict is found in a sequential pass over the parsed
// entries, in file order). Differences: only ASCII whitespace separates
// tokens, and a field or feature beyond int64, or a feature id beyond the
// engine's 2^31-1 columns, is reported as unsupported.
#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <locale.h>
#include <clocale>
#include <cstring>
#include <memory>
#include <sys/mman.h>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "common.cuh"

// An array left uninitialised on allocation, so that its pages are first
// touched by the threads that fill it; arrays of 4 MB and more are mapped
// with transparent huge pages requested (far fewer page faults and TLB misses
// on the hundreds of MB a large file produces).
template <class T>
struct RawBuf {
    T* ptr = nullptr;
    size_t n = 0, bytes = 0;
    bool mapped = false;
    RawBuf() = default;
    RawBuf(const RawBuf&) = delete;
    RawBuf& operator=(const RawBuf&) = delete;
    ~RawBuf() { release(); }
    void alloc(size_t k) {
        release();
        n = k;
        bytes = (k ? k : 1) * sizeof(T);
        if (bytes >= (size_t(4) << 20)) {
            void* m = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1,
                           0);
            if (m != MAP_FAILED) {
                madvise(m, bytes, MADV_HUGEPAGE);  // advisory: ignored where unsupported
                ptr = static_cast<T*>(m);
                mapped = true;
                return;
            }
        }
        ptr = static_cast<T*>(::operator new(bytes));
        mapped = false;
    }
    void release() {
        if (ptr) {
            if (mapped)
                munmap(ptr, bytes);
            else
                ::operator delete(ptr);
        }
        ptr = nullptr;
        n = 0;
    }
    T* data() const { return ptr; }
    T& operator[](size_t i) const { return ptr[i]; }
    size_t size() const { return n; }
};

struct mfm_libffm {
    RawBuf<int64_t> indptr, indices, field_ids;
    RawBuf<double> data, y;
    int64_t n_features = 0;
};

namespace mfm {
namespace {

// Python's str.split() / str.strip() whitespace, ASCII part.
inline bool is_space(unsigned char c) {
    return c == ' ' || (c >= 9 && c <= 13) || (c >= 0x1c && c <= 0x1f);
}

// Python's repr() of a token, for error messages.
std::string py_repr(const char* b, const char* e) {
    const std::string s(b, e);
    const char q = (s.find('\'') != std::string::npos && s.find('"') == std::string::npos) ? '"'
                                                                                          : '\'';
    std::string o(1, q);
    for (unsigned char c : s) {
        if (c == '\\' || c == (unsigned char)q) {
            o.push_back('\\');
            o.push_back((char)c);
        } else if (c == '\t') {
            o += "\\t";
        } else if (c == '\n') {
            o += "\\n";
        } else if (c == '\r') {
            o += "\\r";
        } else if (c < 0x20 || c == 0x7f) {
            char buf[8];
            snprintf(buf, sizeof buf, "\\x%02x", c);
            o += buf;
        } else {
            o.push_back((char)c);
        }
    }
    o.push_back(q);
    return o;
}

enum ParseResult { kParsed, kSyntax, kRange };

inline bool is_digit(char c) { return c >= '0' && c <= '9'; }

// One group of decimal digits with single underscores between digits
// (Python's int() / float() digit groups). Advances p; returns the number of
// digits (0: no group) and whether an underscore was seen.
inline int digit_group(const char*& p, const char* e, bool& underscore) {
    int n = 0;
    while (p < e) {
        if (is_digit(*p)) {
            ++p;
            ++n;
        } else if (*p == '_' && n > 0 && p + 1 < e && is_digit(p[1])) {
            ++p;
            underscore = true;
        } else {
            break;
        }
    }
    return n;
}

// int(token), base 10.
ParseResult parse_int(const char* b, const char* e, int64_t& v) {
    const char* p = b;
    bool neg = false, us = false;
    if (p < e && (*p == '+' || *p == '-')) neg = *p++ == '-';
    const char* d0 = p;
    if (digit_group(p, e, us) == 0 || p != e) return kSyntax;
    uint64_t acc = 0;
    const uint64_t lim = (uint64_t)1 << 63;  // |INT64_MIN|
    for (const char* q = d0; q < e; ++q) {
        if (*q == '_') continue;
        const uint64_t dgt = (uint64_t)(*q - '0');
        if (acc > (lim - dgt) / 10) return kRange;
        acc = acc * 10 + dgt;
    }
    if (!neg && acc == lim) return kRange;
    v = neg ? (int64_t)(0 - acc) : (int64_t)acc;
    return kParsed;
}

// strtod in the "C" locale, whatever the process locale is.
double strtod_c(const char* s, char** end) {
    static locale_t c_loc = newlocale(LC_ALL_MASK, "C", (locale_t)0);
    return strtod_l(s, end, c_loc);
}

// Powers of ten exactly representable in a double (10^0 .. 10^22).
const double kPow10[23] = {1e0,  1e1,  1e2,  1e3,  1e4,  1e5,  1e6,  1e7,
                           1e8,  1e9,  1e10, 1e11, 1e12, 1e13, 1e14, 1e15,
                           1e16, 1e17, 1e18, 1e19, 1e20, 1e21, 1e22};

// float(token). The grammar is checked by hand (Python's float() literal:
// sign, digit groups with an optional fraction and exponent, or inf /
// infinity / nan in any case). The value is exact-rounded either by Clinger's
// fast path (at most 15 significant digits and a power-of-ten scale within
// 10^+-22: one correctly rounded multiply or divide of two exact doubles) or
// by strtod, which rounds correctly; both agree with Python's float().
bool parse_float(const char* b, const char* e, double& v) {
    const char* p = b;
    bool neg = false, us = false;
    if (p < e && (*p == '+' || *p == '-')) neg = *p++ == '-';
    const size_t rest = (size_t)(e - p);
    auto word = [&](const char* w) {
        const size_t n = strlen(w);
        if (rest != n) return false;
        for (size_t i = 0; i < n; ++i)
            if (std::tolower((unsigned char)p[i]) != w[i]) return false;
        return true;
    };
    if (word("inf") || word("infinity")) {
        v = neg ? -HUGE_VAL : HUGE_VAL;
        return true;
    }
    if (word("nan")) {
        v = std::copysign(std::nan(""), neg ? -1.0 : 1.0);
        return true;
    }
    const char* m0 = p;
    const int whole = digit_group(p, e, us);
    const char* w1 = p;
    int frac = 0;
    const char *f0 = p, *f1 = p;
    if (p < e && *p == '.') {
        ++p;
        f0 = p;
        frac = digit_group(p, e, us);
        f1 = p;
    }
    if (whole == 0 && frac == 0) return false;
    const char *x0 = p, *x1 = p;
    if (p < e && (*p == 'e' || *p == 'E')) {
        ++p;
        x0 = p;
        if (p < e && (*p == '+' || *p == '-')) ++p;
        if (digit_group(p, e, us) == 0) return false;
        x1 = p;
    }
    if (p != e) return false;

    // Clinger's fast path
    uint64_t m = 0;
    int sig = 0;  // significant digits kept in m
    bool fits = true;
    auto take = [&](const char* q0, const char* q1) {
        for (const char* q = q0; q < q1; ++q) {
            if (*q == '_') continue;
            if (m == 0 && *q == '0') continue;  // leading zeros
            if (++sig > 15) fits = false;
            m = m * 10 + (uint64_t)(*q - '0');
        }
    };
    take(m0, w1);
    // trailing fraction zeros of an integer-valued mantissa still count as digits
    int fdig = 0;
    for (const char* q = f0; q < f1; ++q) {
        if (*q == '_') continue;
        ++fdig;
        if (m == 0 && *q == '0') continue;
        if (++sig > 15) fits = false;
        m = m * 10 + (uint64_t)(*q - '0');
    }
    long ex = 0;
    if (x1 > x0) {
        const char* q = x0;
        bool eneg = false;
        if (*q == '+' || *q == '-') eneg = *q++ == '-';
        for (; q < x1; ++q) {
            if (*q == '_') continue;
            if (ex < 100000) ex = ex * 10 + (*q - '0');
        }
        if (eneg) ex = -ex;
    }
    const long scale = ex - fdig;
    if (fits && scale >= -22 && scale <= 22) {
        const double dm = (double)m;  // exact: m < 10^15 < 2^53
        v = scale >= 0 ? dm * kPow10[scale] : dm / kPow10[-scale];
        if (neg) v = -v;
        return true;
    }
    // strtod on the token itself (it ends at whitespace, ':' or the buffer's
    // terminating NUL), or on a copy without underscores
    if (!us) {
        char* end = nullptr;
        v = strtod_c(b, &end);
        if (end == e) return true;
    }
    std::string t;
    t.reserve((size_t)(e - b));
    for (const char* q = b; q < e; ++q)
        if (*q != '_') t.push_back(*q);
    v = strtod_c(t.c_str(), nullptr);
    return true;
}

// Calls line(first, last) for every line of [b, e) (Python's universal
// newlines: \n, \r\n, \r); a final line without a terminator counts.
template <class F>
inline void for_each_line(const char* b, const char* e, F&& line) {
    const char* p = b;
    while (p < e) {
        const char* q = p;
        while (q < e && *q != '\n' && *q != '\r') ++q;
        line(p, q);
        if (q < e) q += (*q == '\r' && q + 1 < e && q[1] == '\n') ? 2 : 1;
        p = q;
    }
}

// Splits [b, e) on whitespace (Python's str.split()).
inline void split_tokens(const char* b, const char* e,
                         std::vector<std::pair<const char*, const char*>>& tok) {
    tok.clear();
    for (const char* t = b; t < e;) {
        while (t < e && is_space((unsigned char)*t)) ++t;
        const char* s = t;
        while (t < e && !is_space((unsigned char)*t)) ++t;
        if (t > s) tok.emplace_back(s, t);
    }
}

struct Chunk {
    const char* b = nullptr;
    const char* e = nullptr;
    // counting pass: rows (non-blank lines) and entries (tokens after the
    // label); their prefixes over the chunks place the chunk in the output
    int64_t rows = 0, entries = 0, row0 = 0, entry0 = 0;
    // parsing pass
    int64_t lines = 0;                  // lines read (blank ones included)
    int64_t parsed_rows = 0, parsed_entries = 0;
    int64_t max_feat = -1, max_field = -1;  // over the parsed entries
    // first error: chunk-local line, code, message (with or without the
    // reference's "path:line: " prefix)
    bool err = false, err_prefixed = false;
    int err_code = 0;
    int64_t err_line = 0;
    std::string err_msg;
};

void count_chunk(Chunk& C) {
    std::vector<std::pair<const char*, const char*>> tok;
    for_each_line(C.b, C.e, [&](const char* p, const char* q) {
        split_tokens(p, q, tok);
        if (tok.empty()) return;
        ++C.rows;
        C.entries += (int64_t)tok.size() - 1;
    });
}

// Output slices a chunk parses into (global arrays, the chunk's offsets).
struct Sink {
    int64_t* indptr;    // n_rows + 1: entry offset after each row
    int64_t* indices;   // nnz
    double* data;       // nnz
    int64_t* field;     // nnz (the entry's field, for the file-order pass)
    double* y;          // n_rows
    int64_t* row_line;  // n_rows: chunk-local line of each row
};

void parse_chunk(Chunk& C, const Sink& S) {
    std::vector<std::pair<const char*, const char*>> tok;
    int64_t r = C.row0, k = C.entry0;
    const char* p = C.b;
    while (p < C.e && !C.err) {
        const char* q = p;
        while (q < C.e && *q != '\n' && *q != '\r') ++q;
        const char* line_end = q;
        if (q < C.e) q += (*q == '\r' && q + 1 < C.e && q[1] == '\n') ? 2 : 1;
        ++C.lines;
        split_tokens(p, line_end, tok);
        p = q;
        if (tok.empty()) continue;  // blank line (libffm.py:51-53)
        auto fail_here = [&](int code, bool prefixed, std::string msg) {
            C.err = true;
            C.err_code = code;
            C.err_prefixed = prefixed;
            C.err_line = C.lines;
            C.err_msg = std::move(msg);
        };
        double label;
        if (!parse_float(tok[0].first, tok[0].second, label)) {
            fail_here(MFM_ERR_INVALID, false,
                      "could not convert string to float: " + py_repr(tok[0].first, tok[0].second));
            break;
        }
        S.y[r] = label;
        S.row_line[r] = C.lines;
        for (size_t i = 1; i < tok.size(); ++i) {
            const char *s = tok[i].first, *t = tok[i].second;
            const char* c1 = (const char*)memchr(s, ':', (size_t)(t - s));
            const char* c2 = c1 ? (const char*)memchr(c1 + 1, ':', (size_t)(t - c1 - 1)) : nullptr;
            const bool three = c2 && !memchr(c2 + 1, ':', (size_t)(t - c2 - 1));
            int64_t f = 0, j = 0;
            double x = 0.0;
            ParseResult rf = kSyntax, rj = kSyntax;
            bool ok = three;
            if (ok) {
                rf = parse_int(s, c1, f);
                rj = rf == kSyntax ? kSyntax : parse_int(c1 + 1, c2, j);
                ok = rf != kSyntax && rj != kSyntax && parse_float(c2 + 1, t, x);
            }
            if (!ok) {
                fail_here(MFM_ERR_INVALID, true,
                          "bad token " + py_repr(s, t) + "; expected field:feature:value");
            } else if (rf == kRange || rj == kRange) {
                fail_here(MFM_ERR_UNSUPPORTED, true,
                          "field/feature beyond the int64 range in " + py_repr(s, t));
            } else if (j < 0 || f < 0) {
                fail_here(MFM_ERR_INVALID, true, "negative field/feature in " + py_repr(s, t));
            }
            if (C.err) break;  // the entries before the bad token stay for the file-order pass
            S.indices[k] = j;
            S.field[k] = f;
            S.data[k] = x;
            ++k;
            if (j > C.max_feat) C.max_feat = j;
            if (f > C.max_field) C.max_field = f;
        }
        S.indptr[r + 1] = k;
        ++r;
    }
    C.parsed_rows = r - C.row0;
    C.parsed_entries = k - C.entry0;
}

// The whole file, NUL-terminated (a number at the very end of the file is
// then followed by a byte strtod stops at).
void read_file(const char* path, RawBuf<char>& buf, size_t& size) {
    FILE* fp = fopen(path, "rb");
    if (!fp) fail(MFM_ERR_INVALID, fmt("%s: cannot open (%s)", path, strerror(errno)));
    std::string grow;  // files without a length (pipes) are read in pieces
    long len = -1;
    if (fseek(fp, 0, SEEK_END) == 0) {
        len = ftell(fp);
        fseek(fp, 0, SEEK_SET);
    }
    size = 0;
    if (len >= 0) {
        buf.alloc((size_t)len + 1);
        size_t got;
        while (size < (size_t)len &&
               (got = fread(buf.data() + size, 1, (size_t)len - size, fp)) > 0)
            size += got;
    } else {
        char tmp[1 << 16];
        size_t got;
        while ((got = fread(tmp, 1, sizeof tmp, fp)) > 0) grow.append(tmp, got);
        buf.alloc(grow.size() + 1);
        memcpy(buf.data(), grow.data(), grow.size());
        size = grow.size();
    }
    const bool bad = ferror(fp);
    fclose(fp);
    if (bad) fail(MFM_ERR_INVALID, fmt("%s: read error", path));
    buf[size] = '\0';
}

void read_libffm(const char* path, int n_threads, mfm_libffm& out) {
    RawBuf<char> text;
    size_t text_size = 0;
    read_file(path, text, text_size);
    const char* b = text.data();
    const char* e = b + text_size;
    int nt = n_threads > 0 ? n_threads : (int)std::max(1u, std::thread::hardware_concurrency());
    nt = (int)std::max<int64_t>(1, std::min<int64_t>(nt, (int64_t)text_size / (1 << 20) + 1));
    // chunk boundaries just after a '\n' (a "\r\n" pair is never split)
    std::vector<Chunk> ch(nt);
    const char* at = b;
    for (int c = 0; c < nt; ++c) {
        const char* cut = c + 1 == nt ? e : std::max(at, b + (int64_t)text_size * (c + 1) / nt);
        while (cut < e && cut > b && cut[-1] != '\n') ++cut;
        ch[c].b = at;
        ch[c].e = cut;
        at = cut;
    }
    auto run = [&](auto&& fn) {  // fn(c) on every chunk, one thread each
        std::vector<std::thread> th;
        for (int c = 1; c < nt; ++c) th.emplace_back([&, c] { fn(c); });
        fn(0);
        for (auto& t : th) t.join();
    };
    run([&](int c) { count_chunk(ch[c]); });
    int64_t n_rows = 0, nnz = 0;
    for (Chunk& C : ch) {
        C.row0 = n_rows;
        C.entry0 = nnz;
        n_rows += C.rows;
        nnz += C.entries;
    }
    // the output arrays, sized once; each thread writes (and first touches)
    // only its own slice
    out.indptr.alloc((size_t)n_rows + 1);
    out.indices.alloc((size_t)nnz);
    out.data.alloc((size_t)nnz);
    out.y.alloc((size_t)n_rows);
    RawBuf<int64_t> field, row_line;
    field.alloc((size_t)nnz);
    row_line.alloc((size_t)n_rows);
    out.indptr[0] = 0;
    const Sink S{out.indptr.data(), out.indices.data(), out.data.data(), field.data(),
                 out.y.data(), row_line.data()};
    run([&](int c) { parse_chunk(ch[c], S); });

    // file-order pass: each feature's field (libffm.py:65-69); the first error
    // in file order wins
    int64_t max_feat = -1, max_field = -1;
    for (const Chunk& C : ch) {
        max_feat = std::max(max_feat, C.max_feat);
        max_field = std::max(max_field, C.max_field);
    }
    const bool dense = max_feat < (int64_t(1) << 25);  // else a hash map
    const bool narrow = max_field < INT32_MAX;         // 4-byte table entries
    std::vector<int32_t> fv32(dense && narrow ? (size_t)(max_feat + 1) : 0, -1);
    std::vector<int64_t> fv64(dense && !narrow ? (size_t)(max_feat + 1) : 0, -1);
    std::unordered_map<int64_t, int64_t> fm;
    int64_t line0 = 0;
    for (const Chunk& C : ch) {
        const int64_t k0 = C.entry0, k1 = C.entry0 + C.parsed_entries;
        int64_t bad = -1, prev = -1;  // first conflicting entry and the field seen before
        if (dense && narrow) {
            for (int64_t k = k0; k < k1 && bad < 0; ++k) {
                int32_t& slot = fv32[(size_t)out.indices[(size_t)k]];
                const int32_t f = (int32_t)field[(size_t)k];
                if (slot < 0) slot = f;
                if (slot != f) bad = k, prev = slot;
            }
        } else {
            for (int64_t k = k0; k < k1 && bad < 0; ++k) {
                const int64_t j = out.indices[(size_t)k], f = field[(size_t)k];
                int64_t& slot = dense ? fv64[(size_t)j] : fm.emplace(j, -1).first->second;
                if (slot < 0) slot = f;
                if (slot != f) bad = k, prev = slot;
            }
        }
        if (bad >= 0) {
            // the row holding entry `bad`: the last parsed row starting at or before it
            const int64_t* ip = out.indptr.data();
            const int64_t r = std::upper_bound(ip + C.row0 + 1, ip + C.row0 + C.parsed_rows + 1,
                                               bad) - (ip + 1);
            fail(MFM_ERR_INVALID,
                 fmt("%s:%lld: feature %lld maps to fields %lld and %lld", path,
                     (long long)(line0 + row_line[(size_t)r]), (long long)out.indices[(size_t)bad],
                     (long long)prev, (long long)field[(size_t)bad]));
        }
        if (C.err)
            fail(C.err_code, C.err_prefixed ? fmt("%s:%lld: ", path,
                                                  (long long)(line0 + C.err_line)) + C.err_msg
                                            : C.err_msg);
        line0 += C.lines;
    }
    if (max_feat >= INT32_MAX)
        fail(MFM_ERR_UNSUPPORTED, fmt("%s: feature %lld exceeds the engine's 2^31-1 columns", path,
                                      (long long)max_feat));
    out.n_features = max_feat + 1;
    out.field_ids.alloc((size_t)out.n_features);
    std::fill(out.field_ids.data(), out.field_ids.data() + out.n_features, int64_t(0));
    if (dense && narrow) {
        for (int64_t j = 0; j < out.n_features; ++j)
            if (fv32[(size_t)j] >= 0) out.field_ids[(size_t)j] = fv32[(size_t)j];
    } else if (dense) {
        for (int64_t j = 0; j < out.n_features; ++j)
            if (fv64[(size_t)j] >= 0) out.field_ids[(size_t)j] = fv64[(size_t)j];
    } else {
        for (const auto& kv : fm) out.field_ids[(size_t)kv.first] = kv.second;
    }
}

}  // namespace
}  // namespace mfm

using namespace mfm;

extern "C" int mfm_libffm_read(const char* path, int n_threads, mfm_libffm** out) {
    return guarded([&] {
        if (!path || !out) fail(MFM_ERR_INVALID, "path and out must be provided");
        *out = nullptr;
        auto* f = new mfm_libffm();
        try {
            read_libffm(path, n_threads, *f);
        } catch (...) {
            delete f;
            throw;
        }
        *out = f;
    });
}

extern "C" int mfm_libffm_info(const mfm_libffm* f, int64_t* n_rows, int64_t* nnz,
                               int64_t* n_features) {
    return guarded([&] {
        if (!f) fail(MFM_ERR_INVALID, "no libffm handle");
        if (n_rows) *n_rows = (int64_t)f->y.size();
        if (nnz) *nnz = (int64_t)f->indices.size();
        if (n_features) *n_features = f->n_features;
    });
}

extern "C" int mfm_libffm_arrays(const mfm_libffm* f, const int64_t** indptr,
                                 const int64_t** indices, const double** data, const double** y,
                                 const int64_t** field_ids) {
    return guarded([&] {
        if (!f) fail(MFM_ERR_INVALID, "no libffm handle");
        if (indptr) *indptr = f->indptr.data();
        if (indices) *indices = f->indices.data();
        if (data) *data = f->data.data();
        if (y) *y = f->y.data();
        if (field_ids) *field_ids = f->field_ids.data();
    });
}

extern "C" void mfm_libffm_free(mfm_libffm* f) { delete f; }
