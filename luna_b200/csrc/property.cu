// property.cu -- VNN-LIB properties: the text front end, the per-box
// verdict (host and device) and bounding a batch of boxes against a property
// (extern "C" entry points declared in include/luna_b200.h).
//
// The parser reproduces what Luna reads from a property file, including how
// it reads unusual files: Luna walks a flat token list with one cursor and
// per-construct skipping rules, and where a file nests beyond what those
// rules expect (an arithmetic expression inside an input bound, an OR
// inside an OR branch) the cursor lands somewhere Luna's own later rules
// then interpret.  The rules are therefore kept as cursor moves over the
// token list (VnnLibInputParser.cpp:120-372 for input bounds, :374-928 for
// output constraints) rather than as a tree walk, which would read such
// files differently.
#include "handle.h"
#include "property.cuh"

#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

struct lb200_property {
    int64_t n_in = 0, n_out = 0;
    std::vector<float> lower, upper;  // [n_in]
    int64_t nspec = 0;
    std::vector<float> C;             // [nspec, n_out]
    std::vector<float> thr;           // [nspec]
    std::vector<int32_t> branch;      // [nspec]
    int32_t n_branches = 0;
    bool spec_dropped = false;
    std::string spec_error;
};

namespace {

using Tokens = std::vector<std::string>;

// ------------------------------------------------------------------ text
// VnnLibInputParser::readVnnlibFile (:1131-1164): lines split on '\n',
// trimmed of ' ', '\r', '\n' (not tabs), blank lines and lines whose first
// character is ';' dropped, the rest concatenated with no separator.
std::string joined_lines(const char* text, size_t len) {
    std::string out;
    size_t a = 0;
    while (a < len) {
        size_t b = a;
        while (b < len && text[b] != '\n') ++b;
        size_t s = a, e = b;
        auto blank = [](char c) { return c == ' ' || c == '\r' || c == '\n'; };
        while (s < e && blank(text[s])) ++s;
        while (e > s && blank(text[e - 1])) --e;
        if (e > s && text[s] != ';') out.append(text + s, e - s);
        a = b + 1;
    }
    return out;
}

// VnnLibInputParser::tokenize (:1166-1183): the leftmost match of
// "(" | ")" | [A-Za-z0-9_\-\\.]+ | "<=" | ">=" | "+" | "-" | "*", first
// alternative winning; characters no alternative matches are dropped.
bool word_char(char c) {
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' || c == '-' ||
           c == '\\' || c == '.';
}

Tokens tokenize(const std::string& s) {
    Tokens t;
    size_t i = 0;
    while (i < s.size()) {
        const char c = s[i];
        if (c == '(' || c == ')') {
            t.emplace_back(1, c);
            ++i;
        } else if (word_char(c)) {
            size_t j = i;
            while (j < s.size() && word_char(s[j])) ++j;
            t.emplace_back(s, i, j - i);
            i = j;
        } else if ((c == '<' || c == '>') && i + 1 < s.size() && s[i + 1] == '=') {
            t.emplace_back(s, i, 2);
            i += 2;
        } else if (c == '+' || c == '*') {
            t.emplace_back(1, c);
            ++i;
        } else {
            ++i;
        }
    }
    return t;
}

// -------------------------------------------------------------- variables
// Name "P_k": the name split on '_' with empty pieces dropped (strtok) must
// give exactly two pieces, the first being P (:1185-1192, :372-379).
bool is_var(const std::string& name, char prefix) {
    std::vector<std::string> parts;
    size_t i = 0;
    while (i < name.size()) {
        while (i < name.size() && name[i] == '_') ++i;
        size_t j = i;
        while (j < name.size() && name[j] != '_') ++j;
        if (j > i) parts.emplace_back(name, i, j - i);
        i = j;
    }
    return parts.size() == 2 && parts[0].size() == 1 && parts[0][0] == prefix;
}

// The index of a variable accepted by is_var (:1194-1215): its second piece
// must be all digits.
int64_t var_index(const std::string& name) {
    size_t i = 0;
    while (name[i] == '_') ++i;
    ++i;  // the prefix letter
    while (name[i] == '_') ++i;
    size_t j = i;
    while (j < name.size() && name[j] != '_') ++j;
    if (j == i) throw std::runtime_error("Invalid variable name format: " + name);
    int64_t v = 0;
    for (size_t k = i; k < j; ++k) {
        if (name[k] < '0' || name[k] > '9') throw std::runtime_error("Invalid variable index in: " + name);
        v = v * 10 + (name[k] - '0');
        // Luna's atoi has no defined result past INT_MAX; refuse such names.
        if (v > std::numeric_limits<int32_t>::max()) throw std::runtime_error("variable index too large: " + name);
    }
    return v;
}

// The number a token spells (:20-30, std::stod): strtod must consume it all.
double scalar(const std::string& tok) {
    errno = 0;
    char* end = nullptr;
    const double v = std::strtod(tok.c_str(), &end);
    if (end == tok.c_str()) throw std::invalid_argument("stod: no conversion of '" + tok + "'");
    if (errno == ERANGE) throw std::out_of_range("stod: '" + tok + "' is out of range");
    if (end != tok.c_str() + tok.size()) throw std::runtime_error("'" + tok + "' is not a valid scalar");
    return v;
}

// The output-side test for a numeric literal (:381-430): optional leading
// '-', digits with at most one '.', and an optional exponent that needs a
// digit before it, a character after it, and only digits after its sign.
bool looks_scalar(const std::string& t) {
    if (t.empty()) return false;
    size_t k = 0;
    if (t[0] == '-') {
        if (t.size() == 1) return false;
        k = 1;
    }
    bool dot = false, digit = false;
    for (; k < t.size(); ++k) {
        const char c = t[k];
        if (c == '.') {
            if (dot) return false;
            dot = true;
        } else if (c >= '0' && c <= '9') {
            digit = true;
        } else if (c == 'e' || c == 'E') {
            if (!digit || k + 1 >= t.size()) return false;
            size_t e = k + 1;
            if (t[e] == '-' || t[e] == '+') ++e;
            for (; e < t.size(); ++e)
                if (t[e] < '0' || t[e] > '9') return false;
            return true;
        } else {
            return false;
        }
    }
    return digit;
}

bool is_and(const std::string& s) { return s == "and" || s == "AND" || s == "And"; }
bool is_or(const std::string& s) { return s == "or" || s == "OR" || s == "Or"; }
bool is_cmp(const std::string& s) { return s == "<=" || s == ">="; }

// ---------------------------------------------------------------- cursor
struct Cursor {
    const Tokens& t;
    size_t i = 0;
    explicit Cursor(const Tokens& tok) : t(tok) {}
    bool end() const { return i >= t.size(); }
    bool at(const char* s) const { return i < t.size() && t[i] == s; }
    // Advance to the next ")" and step over it.
    void past_close() {
        while (i < t.size() && t[i] != ")") ++i;
        ++i;
    }
    // From just inside an open "(", advance past its balanced ")".
    void past_balanced() {
        int depth = 1;
        while (i < t.size() && depth > 0) {
            if (t[i] == "(") ++depth;
            else if (t[i] == ")") --depth;
            ++i;
        }
    }
    // The top-level loop shared by both passes: each "(" opens a command
    // handled by `cmd`, which leaves the cursor on the command's ")" (stepped
    // over here) or wherever its rules stop; other tokens are skipped.
    template <class F>
    void commands(F&& cmd) {
        while (i < t.size()) {
            if (t[i] == "(") {
                ++i;
                cmd();
                if (at(")")) ++i;
            } else {
                ++i;
            }
        }
    }
};

// ----------------------------------------------------------- input bounds
struct InputBound {
    double lo = -std::numeric_limits<double>::infinity();
    double hi = std::numeric_limits<double>::infinity();
};

struct InputPass {
    Cursor c;
    int64_t n_in;
    std::vector<InputBound> b;
    InputPass(const Tokens& t, int64_t n) : c(t), n_in(n), b((size_t)n) {}

    InputBound* slot(int64_t k) { return k < n_in ? &b[(size_t)k] : nullptr; }

    // A bound "(<= X_k v)", "(<= v X_k)", or ">=" forms (:237-331).
    void bound(const std::string& op) {
        ++c.i;
        if (c.i + 1 >= c.t.size()) return;
        const std::string& a = c.t[c.i];
        const std::string& v = c.t[c.i + 1];
        bool var_first;
        if (is_var(a, 'X')) var_first = true;
        else if (is_var(v, 'X')) var_first = false;
        else {
            c.i += 2;
            c.past_close();
            return;
        }
        const int64_t k = var_index(var_first ? a : v);
        const double value = scalar(var_first ? v : a);
        const bool upper = (op == "<=") == var_first;
        if (InputBound* s = slot(k)) (upper ? s->hi : s->lo) = value;
        c.i += 2;
        c.past_close();
    }

    // From the operator after "(" (:207-335).
    void condition() {
        if (c.end()) return;
        const std::string& op = c.t[c.i];
        if (is_and(op) || is_or(op)) {
            ++c.i;
            while (!c.end() && !c.at(")")) {
                if (c.at("(")) {
                    ++c.i;
                    condition();
                } else {
                    ++c.i;
                }
            }
            ++c.i;
        } else if (is_cmp(op)) {
            bound(op);
        } else {
            c.past_close();
        }
    }

    void command() {
        if (c.end()) return;
        const std::string& cmd = c.t[c.i];
        if (cmd == "declare-const") {
            // "(declare-const X_k Real)" names an input (:154-183); the
            // cursor stops after the type.
            ++c.i;
            if (c.i + 1 >= c.t.size()) return;
            const std::string& name = c.t[c.i];
            const bool real = c.t[c.i + 1] == "Real";
            if (real && is_var(name, 'X')) (void)var_index(name);
            c.i += 2;
        } else if (cmd == "assert") {
            ++c.i;
            if (c.at("(")) {
                ++c.i;
                condition();
            }
        } else {
            ++c.i;
            c.past_balanced();
            --c.i;
        }
    }

    void run() { c.commands([this] { command(); }); }
};

// ----------------------------------------------------- output constraints
struct Term {
    int64_t out;
    double coef;
};
struct Row {  // sum coef * Y <= thr
    std::vector<Term> terms;
    double thr = 0.0;
};

struct OutputPass {
    Cursor c;
    std::vector<Row> rows;                     // top-level constraints
    std::vector<std::vector<Row>> branches;    // OR branches
    bool has_or = false;
    explicit OutputPass(const Tokens& t) : c(t) {}

    // A linear expression (:432-631): a Y_k, a literal, or "(+ ...)",
    // "(- a [b])" (a unary minus keeps its operand's sign, as Luna reads it),
    // "(* ...)" (literals multiply; the last Y_k named takes the product; a
    // nested expression takes the product so far, which then restarts).
    void expr(std::vector<Term>& terms, double& sum) {
        if (c.end()) return;
        const std::string& tok = c.t[c.i];
        if (is_var(tok, 'Y')) {
            terms.push_back({var_index(tok), 1.0});
            ++c.i;
            return;
        }
        if (looks_scalar(tok)) {
            sum += scalar(tok);
            ++c.i;
            return;
        }
        if (tok != "(") {
            ++c.i;
            return;
        }
        ++c.i;
        if (c.end()) return;
        const std::string op = c.t[c.i];
        ++c.i;
        if (op == "+") {
            while (!c.end() && !c.at(")")) expr(terms, sum);
            if (c.at(")")) ++c.i;
        } else if (op == "-") {
            // Each operand's literals are summed on their own first, and
            // that sum then added (or subtracted): the same roundings as Luna.
            double s1 = 0.0;
            expr(terms, s1);
            sum += s1;
            if (!c.end() && !c.at(")")) {
                std::vector<Term> sub;
                double s2 = 0.0;
                expr(sub, s2);
                for (Term& x : sub) terms.push_back({x.out, -x.coef});
                sum -= s2;
            }
            while (!c.end() && !c.at(")")) ++c.i;
            if (c.at(")")) ++c.i;
        } else if (op == "*") {
            double k = 1.0;
            int64_t var = -1;
            while (!c.end() && !c.at(")")) {
                const std::string& s = c.t[c.i];
                if (looks_scalar(s)) {
                    k *= scalar(s);
                    ++c.i;
                } else if (is_var(s, 'Y')) {
                    var = var_index(s);
                    ++c.i;
                } else if (s == "(") {
                    std::vector<Term> sub;
                    double s2 = 0.0;
                    expr(sub, s2);
                    for (Term& x : sub) terms.push_back({x.out, x.coef * k});
                    sum += s2 * k;
                    k = 1.0;
                    var = -1;
                } else {
                    ++c.i;
                }
            }
            if (var >= 0) terms.push_back({var, k});
            if (c.at(")")) ++c.i;
        } else {
            c.past_balanced();
        }
    }

    // One side of a comparison (:690-735).
    void side(std::vector<Term>& terms, double& sum) {
        const std::string& tok = c.t[c.i];
        if (tok == "(") {
            expr(terms, sum);
        } else if (is_var(tok, 'Y')) {
            terms.push_back({var_index(tok), 1.0});
            ++c.i;
        } else if (looks_scalar(tok)) {
            sum = scalar(tok);
            ++c.i;
        } else {
            ++c.i;
        }
    }

    // "(<= lhs rhs)" or ">=" normalised to sum coef * Y <= thr (:679-770);
    // nothing is recorded without an output variable.
    void comparison(const std::string& op, std::vector<Row>& into) {
        ++c.i;
        if (c.end()) return;
        std::vector<Term> lt, rt;
        double ls = 0.0, rs = 0.0;
        side(lt, ls);
        if (!c.end() && !c.at(")")) side(rt, rs);
        if (!lt.empty() || !rt.empty()) {
            Row r;
            r.terms = lt;
            for (Term& x : rt) r.terms.push_back({x.out, -x.coef});
            r.thr = rs - ls;
            if (op == ">=") {
                for (Term& x : r.terms) x.coef = -x.coef;
                r.thr = -r.thr;
            }
            into.push_back(std::move(r));
        }
        c.past_close();
    }

    // Inside one OR branch (:773-915): conjunctions and comparisons; any
    // other construct is skipped to its first ")".
    void branch(std::vector<Row>& into) {
        if (c.end()) return;
        const std::string& op = c.t[c.i];
        if (is_and(op)) {
            ++c.i;
            while (!c.end() && !c.at(")")) {
                if (c.at("(")) {
                    ++c.i;
                    branch(into);
                } else {
                    ++c.i;
                }
            }
            ++c.i;
        } else if (is_cmp(op)) {
            comparison(op, into);
        } else {
            c.past_close();
        }
    }

    // From the operator after "(" (:633-771).
    void condition() {
        if (c.end()) return;
        const std::string& op = c.t[c.i];
        if (is_and(op)) {
            ++c.i;
            while (!c.end() && !c.at(")")) {
                if (c.at("(")) {
                    ++c.i;
                    condition();
                } else {
                    ++c.i;
                }
            }
            ++c.i;
        } else if (is_or(op)) {
            ++c.i;
            std::vector<std::vector<Row>> found;
            while (!c.end() && !c.at(")")) {
                if (c.at("(")) {
                    ++c.i;
                    std::vector<Row> b;
                    branch(b);
                    if (!b.empty()) found.push_back(std::move(b));
                } else {
                    ++c.i;
                }
            }
            for (auto& b : found) branches.push_back(std::move(b));
            if (!found.empty()) has_or = true;
            ++c.i;
        } else if (is_cmp(op)) {
            comparison(op, rows);
        } else {
            c.past_close();
        }
    }

    void command() {
        if (c.end()) return;
        if (c.t[c.i] == "assert") {
            ++c.i;
            if (c.at("(")) {
                ++c.i;
                condition();
            }
        } else {
            ++c.i;
            c.past_balanced();
            --c.i;
        }
    }

    void run() { c.commands([this] { command(); }); }
};

// OutputConstraintSet::toCMatrix (OutputConstraint.cpp:71-173): with any OR
// branch the rows are the branches' rows in order (top-level constraints
// are then not used); otherwise the top-level constraints.  Each term
// stores its coefficient into its column (a later term of the same column
// replaces an earlier one).
void to_spec(const OutputPass& o, lb200_property& p) {
    std::vector<const Row*> rows;
    std::vector<int32_t> br;
    if (o.has_or) {
        for (size_t b = 0; b < o.branches.size(); ++b)
            for (const Row& r : o.branches[b]) {
                rows.push_back(&r);
                br.push_back((int32_t)b);
            }
    } else {
        for (const Row& r : o.rows) {
            rows.push_back(&r);
            br.push_back(0);
        }
    }
    if (rows.empty()) return;  // no constraints: Luna sets no specification
    std::vector<float> C(rows.size() * (size_t)p.n_out, 0.f), thr(rows.size());
    for (size_t r = 0; r < rows.size(); ++r) {
        for (const Term& x : rows[r]->terms) {
            if (x.out >= p.n_out)
                throw std::runtime_error("Output index " + std::to_string(x.out) + " exceeds output dimension " +
                                         std::to_string(p.n_out));
            C[r * (size_t)p.n_out + (size_t)x.out] = (float)x.coef;
        }
        thr[r] = (float)rows[r]->thr;
    }
    p.nspec = (int64_t)rows.size();
    p.C = std::move(C);
    p.thr = std::move(thr);
    p.branch = std::move(br);
    p.n_branches = o.has_or ? (int32_t)o.branches.size() : 0;
}

__global__ void property_status_kernel(const float* __restrict__ lb, const float* __restrict__ ub, int64_t n_boxes,
                                       int64_t nspec, const float* __restrict__ thr, const int32_t* __restrict__ branch,
                                       int32_t n_branches, int32_t* __restrict__ status) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_boxes) return;
    status[b] = lb200::box_status(lb + b * nspec, ub + b * nspec, thr, branch, nspec, n_branches);
}

void launch_status(const float* lb, const float* ub, int64_t n_boxes, int64_t nspec, const float* thr,
                   const int32_t* branch, int32_t n_branches, int32_t* status, cudaStream_t s) {
    if (n_boxes <= 0) return;
    const unsigned blocks = (unsigned)((n_boxes + 255) / 256);
    property_status_kernel<<<blocks, 256, 0, s>>>(lb, ub, n_boxes, nspec, thr, branch, n_branches, status);
    LB_CUDA(cudaGetLastError());
}

void check_branches(const int32_t* branch, int64_t nspec, int32_t n_branches) {
    if (n_branches <= 0) return;
    if (!branch) throw std::invalid_argument("branch_of_row is required with n_branches > 0");
    for (int64_t r = 0; r < nspec; ++r)
        if (branch[r] < 0 || branch[r] >= n_branches)
            throw std::invalid_argument("Branch ID " + std::to_string(branch[r]) + " out of range [0, " +
                                        std::to_string(n_branches) + ")");
}

// The property's specification on the model's device, ordered on s: C
// [rows, n_out] (the identity when the property has none, as Luna's
// OutputConstraintSet::identityC), and with a specification its thresholds
// and the branch of each row.
struct DeviceSpec {
    float* C = nullptr;
    float* thr = nullptr;
    int32_t* branch = nullptr;
    int64_t rows = 0;
};

DeviceSpec stage_spec(lb200::Model& m, const lb200_property* prop, cudaStream_t s) {
    if (prop->n_in != m.n_in() || prop->n_out != m.n_out())
        throw std::invalid_argument("the property was parsed for " + std::to_string(prop->n_in) + " inputs / " +
                                    std::to_string(prop->n_out) + " outputs, the model has " +
                                    std::to_string(m.n_in()) + " / " + std::to_string(m.n_out()));
    const bool spec = prop->nspec > 0;
    const int64_t nout = m.n_out();
    DeviceSpec d;
    d.rows = spec ? prop->nspec : nout;
    d.C = m.staging("io_C", (size_t)d.rows * nout);
    std::vector<float> eye;
    const float* C = prop->C.data();
    if (!spec) {
        eye.assign((size_t)nout * nout, 0.f);
        for (int64_t k = 0; k < nout; ++k) eye[(size_t)(k * nout + k)] = 1.f;
        C = eye.data();
    }
    // Pageable sources: each copy has left the host buffer when it returns.
    LB_CUDA(cudaMemcpyAsync(d.C, C, (size_t)d.rows * nout * 4, cudaMemcpyHostToDevice, s));
    if (spec) {
        d.thr = m.staging("io_thr", (size_t)d.rows);
        d.branch = reinterpret_cast<int32_t*>(m.staging("io_branch", (size_t)d.rows));
        LB_CUDA(cudaMemcpyAsync(d.thr, prop->thr.data(), d.rows * 4, cudaMemcpyHostToDevice, s));
        LB_CUDA(cudaMemcpyAsync(d.branch, prop->branch.data(), d.rows * 4, cudaMemcpyHostToDevice, s));
    }
    return d;
}

template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        return lb200::set_last_error(e.what());
    } catch (...) {
        return lb200::set_last_error("unknown error");
    }
}

}  // namespace

extern "C" {

int lb200_property_parse(const char* text, int64_t len, int64_t n_in, int64_t n_out, lb200_property** out) {
    if (!out) return lb200::set_last_error("lb200_property_parse: null output");
    *out = nullptr;
    if (!text && len > 0) return lb200::set_last_error("lb200_property_parse: null text");
    if (len < 0 || n_in <= 0 || n_out <= 0) return lb200::set_last_error("lb200_property_parse: bad sizes");
    return guard([&] {
        const Tokens tok = tokenize(joined_lines(text, (size_t)len));
        auto* p = new lb200_property;
        try {
            p->n_in = n_in;
            p->n_out = n_out;
            InputPass in(tok, n_in);
            try {
                in.run();
            } catch (const std::exception& e) {
                throw std::runtime_error(std::string("Failed to parse VNN-LIB input bounds: ") + e.what());
            }
            p->lower.resize((size_t)n_in);
            p->upper.resize((size_t)n_in);
            for (int64_t k = 0; k < n_in; ++k) {
                p->lower[(size_t)k] = (float)in.b[(size_t)k].lo;
                p->upper[(size_t)k] = (float)in.b[(size_t)k].hi;
            }
            // Output constraints that fail to parse or convert are dropped
            // (TorchModelOnnxFactory.cpp:177-182).
            try {
                OutputPass o(tok);
                o.run();
                to_spec(o, *p);
            } catch (const std::exception& e) {
                p->nspec = 0;
                p->C.clear();
                p->thr.clear();
                p->branch.clear();
                p->n_branches = 0;
                p->spec_dropped = true;
                p->spec_error = e.what();
            }
        } catch (...) {
            delete p;
            throw;
        }
        *out = p;
    });
}

int lb200_property_get_info(const lb200_property* p, lb200_property_info* info) {
    if (!p || !info) return lb200::set_last_error("lb200_property_get_info: null argument");
    std::memset(info, 0, sizeof *info);
    info->n_in = p->n_in;
    info->n_out = p->n_out;
    info->nspec = p->nspec;
    info->n_branches = p->n_branches;
    info->spec_dropped = p->spec_dropped ? 1 : 0;
    std::strncpy(info->spec_error, p->spec_error.c_str(), sizeof info->spec_error - 1);
    return 0;
}

int lb200_property_input_box(const lb200_property* p, float* lower, float* upper) {
    if (!p) return lb200::set_last_error("lb200_property_input_box: null property");
    if (lower) std::memcpy(lower, p->lower.data(), p->lower.size() * 4);
    if (upper) std::memcpy(upper, p->upper.data(), p->upper.size() * 4);
    return 0;
}

int lb200_property_spec(const lb200_property* p, float* C, float* thresholds, int32_t* branch_of_row) {
    if (!p) return lb200::set_last_error("lb200_property_spec: null property");
    if (C && !p->C.empty()) std::memcpy(C, p->C.data(), p->C.size() * 4);
    if (thresholds && !p->thr.empty()) std::memcpy(thresholds, p->thr.data(), p->thr.size() * 4);
    if (branch_of_row && !p->branch.empty()) std::memcpy(branch_of_row, p->branch.data(), p->branch.size() * 4);
    return 0;
}

void lb200_property_free(lb200_property* p) { delete p; }

int lb200_property_status(const float* lb, const float* ub, int64_t n_boxes, int64_t nspec, const float* thresholds,
                          const int32_t* branch_of_row, int32_t n_branches, int32_t* status) {
    if (n_boxes < 0 || nspec < 0) return lb200::set_last_error("lb200_property_status: bad sizes");
    if (n_boxes > 0 && (!status || (nspec > 0 && (!lb || !ub || !thresholds))))
        return lb200::set_last_error("lb200_property_status: null buffer");
    return guard([&] {
        check_branches(branch_of_row, nspec, n_branches);
        for (int64_t b = 0; b < n_boxes; ++b)
            status[b] = lb200::box_status(lb + b * nspec, ub + b * nspec, thresholds, branch_of_row, nspec, n_branches);
    });
}

int lb200_property_status_device(const float* d_lb, const float* d_ub, int64_t n_boxes, int64_t nspec,
                                 const float* d_thresholds, const int32_t* d_branch_of_row, int32_t n_branches,
                                 int32_t* d_status, void* stream) {
    if (n_boxes < 0 || nspec < 0) return lb200::set_last_error("lb200_property_status_device: bad sizes");
    if (n_boxes > 0 && (!d_status || (nspec > 0 && (!d_lb || !d_ub || !d_thresholds))))
        return lb200::set_last_error("lb200_property_status_device: null buffer");
    if (n_branches > 0 && !d_branch_of_row)
        return lb200::set_last_error("lb200_property_status_device: branch_of_row is required with n_branches > 0");
    return guard([&] {
        launch_status(d_lb, d_ub, n_boxes, nspec, d_thresholds, d_branch_of_row, n_branches, d_status,
                      static_cast<cudaStream_t>(stream));
    });
}

int lb200_compute_property(lb200_model* model, int method, const lb200_property* prop, const float* x_lower,
                           const float* x_upper, int64_t n_boxes, float* out_lb, float* out_ub, int32_t* status,
                           lb200_stats* stats) {
    if (!model || !prop) return lb200::set_last_error("lb200_compute_property: null model or property");
    if ((x_lower == nullptr) != (x_upper == nullptr))
        return lb200::set_last_error("lb200_compute_property: give both box arrays or neither");
    if (!x_lower && n_boxes != 1)
        return lb200::set_last_error("lb200_compute_property: the property's own box is one box (n_boxes = 1)");
    if (n_boxes < 0) return lb200::set_last_error("lb200_compute_property: bad sizes");
    if (n_boxes > 0 && (!out_lb || !out_ub)) return lb200::set_last_error("lb200_compute_property: null buffer");
    return guard([&] {
        lb200::Model& m = *model->m;
        LB_CUDA(cudaSetDevice(m.device()));
        cudaStream_t s = model->stream;
        const DeviceSpec d = stage_spec(m, prop, s);
        if (n_boxes == 0) return;
        const float* xl = x_lower ? x_lower : prop->lower.data();
        const float* xu = x_upper ? x_upper : prop->upper.data();
        const bool spec = prop->nspec > 0;
        const size_t nx = (size_t)n_boxes * m.n_in();
        const size_t no = (size_t)n_boxes * d.rows;
        float* dxl = m.staging("io_xl", nx);
        float* dxu = m.staging("io_xu", nx);
        float* dlb = m.staging("io_lb", no);
        float* dub = m.staging("io_ub", no);
        LB_CUDA(cudaMemcpyAsync(dxl, xl, nx * 4, cudaMemcpyHostToDevice, s));
        LB_CUDA(cudaMemcpyAsync(dxu, xu, nx * 4, cudaMemcpyHostToDevice, s));
        int32_t* dst = (spec && status) ? reinterpret_cast<int32_t*>(m.staging("io_status", (size_t)n_boxes)) : nullptr;
        // Luna's CLI calls compute_bounds(..., COMPUTE_LOWER, COMPUTE_UPPER),
        // both on by default.
        m.compute(method, dxl, dxu, n_boxes, d.C, 1, d.rows, d.thr, true, true, dlb, dub, s, stats, d.branch,
                  prop->n_branches);
        LB_CUDA(cudaMemcpyAsync(out_lb, dlb, no * 4, cudaMemcpyDeviceToHost, s));
        LB_CUDA(cudaMemcpyAsync(out_ub, dub, no * 4, cudaMemcpyDeviceToHost, s));
        if (dst) {
            launch_status(dlb, dub, n_boxes, d.rows, d.thr, d.branch, prop->n_branches, dst, s);
            LB_CUDA(cudaMemcpyAsync(status, dst, (size_t)n_boxes * 4, cudaMemcpyDeviceToHost, s));
        }
        LB_CUDA(cudaStreamSynchronize(s));
        if (status && !spec)
            for (int64_t b = 0; b < n_boxes; ++b) status[b] = LB200_STATUS_UNKNOWN;
    });
}

int lb200_compute_property_device(lb200_model* model, int method, const lb200_property* prop,
                                  const float* d_x_lower, const float* d_x_upper, int64_t n_boxes, float* d_out_lb,
                                  float* d_out_ub, int32_t* d_status, void* stream, lb200_stats* stats) {
    if (!model || !prop) return lb200::set_last_error("lb200_compute_property_device: null model or property");
    if (n_boxes < 0) return lb200::set_last_error("lb200_compute_property_device: bad sizes");
    if (n_boxes > 0 && (!d_x_lower || !d_x_upper || !d_out_lb || !d_out_ub))
        return lb200::set_last_error("lb200_compute_property_device: null buffer");
    return guard([&] {
        lb200::Model& m = *model->m;
        LB_CUDA(cudaSetDevice(m.device()));
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const DeviceSpec d = stage_spec(m, prop, s);
        if (n_boxes == 0) return;
        m.compute(method, d_x_lower, d_x_upper, n_boxes, d.C, 1, d.rows, d.thr, true, true, d_out_lb, d_out_ub, s,
                  stats, d.branch, prop->n_branches);
        if (d_status) {
            if (prop->nspec > 0)
                launch_status(d_out_lb, d_out_ub, n_boxes, d.rows, d.thr, d.branch, prop->n_branches, d_status, s);
            else
                LB_CUDA(cudaMemsetAsync(d_status, 0, (size_t)n_boxes * 4, s));  // LB200_STATUS_UNKNOWN
        }
        LB_CUDA(cudaStreamSynchronize(s));
    });
}

}  // extern "C"
