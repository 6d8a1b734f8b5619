// profile.cpp -- profile JSON loading and validation (host side).
//
// A small recursive-descent JSON reader (objects, arrays, strings, numbers,
// true/false/null) is enough for the flat media profiles; numbers keep their
// literal text so 64-bit integers are read exactly.
#include "profile.h"

#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <fstream>
#include <limits>
#include <map>
#include <memory>
#include <sstream>
#include <vector>

namespace hbfb {
namespace {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool boolean = false;
    std::string text;  // number literal or string value
    std::vector<Json> items;
    std::map<std::string, Json> fields;
};

class Reader {
  public:
    explicit Reader(const std::string& s) : s_(s) {}
    bool parse(Json* out)
    {
        if (!value(out, 0)) return false;
        ws();
        return i_ == s_.size();
    }

  private:
    void ws()
    {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' ||
                                  s_[i_] == '\t' || s_[i_] == '\r'))
            ++i_;
    }
    bool literal(const char* word)
    {
        const std::string w(word);
        if (s_.compare(i_, w.size(), w) != 0) return false;
        i_ += w.size();
        return true;
    }
    bool string(std::string* out)
    {
        if (i_ >= s_.size() || s_[i_] != '"') return false;
        ++i_;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size()) return false;
                const char e = s_[i_++];
                switch (e) {
                case 'n': c = '\n'; break;
                case 't': c = '\t'; break;
                case 'r': c = '\r'; break;
                case 'b': c = '\b'; break;
                case 'f': c = '\f'; break;
                case 'u':
                    if (i_ + 4 > s_.size()) return false;
                    i_ += 4;
                    c = '?';
                    break;
                default: c = e; break;
                }
            }
            out->push_back(c);
        }
        if (i_ >= s_.size()) return false;
        ++i_;
        return true;
    }
    bool value(Json* out, int depth)
    {
        if (depth > 64) return false;
        ws();
        if (i_ >= s_.size()) return false;
        const char c = s_[i_];
        if (c == '{') {
            ++i_;
            out->kind = Json::Object;
            ws();
            if (i_ < s_.size() && s_[i_] == '}') { ++i_; return true; }
            for (;;) {
                ws();
                std::string key;
                if (!string(&key)) return false;
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') return false;
                ++i_;
                Json v;
                if (!value(&v, depth + 1)) return false;
                if (out->fields.count(key)) return false;  // duplicate key
                out->fields.emplace(key, std::move(v));
                ws();
                if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
                if (i_ < s_.size() && s_[i_] == '}') { ++i_; return true; }
                return false;
            }
        }
        if (c == '[') {
            ++i_;
            out->kind = Json::Array;
            ws();
            if (i_ < s_.size() && s_[i_] == ']') { ++i_; return true; }
            for (;;) {
                Json v;
                if (!value(&v, depth + 1)) return false;
                out->items.push_back(std::move(v));
                ws();
                if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
                if (i_ < s_.size() && s_[i_] == ']') { ++i_; return true; }
                return false;
            }
        }
        if (c == '"') {
            out->kind = Json::String;
            return string(&out->text);
        }
        if (literal("true")) { out->kind = Json::Bool; out->boolean = true; return true; }
        if (literal("false")) { out->kind = Json::Bool; return true; }
        if (literal("null")) { out->kind = Json::Null; return true; }
        const std::size_t b = i_;
        while (i_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[i_])) ||
                                  s_[i_] == '-' || s_[i_] == '+' || s_[i_] == '.' ||
                                  s_[i_] == 'e' || s_[i_] == 'E'))
            ++i_;
        if (i_ == b) return false;
        out->kind = Json::Number;
        out->text = s_.substr(b, i_ - b);
        return true;
    }
    const std::string& s_;
    std::size_t i_ = 0;
};

struct FieldError {
    std::string message;
};

const Json& need(const Json& obj, const char* key)
{
    const auto it = obj.fields.find(key);
    if (it == obj.fields.end())
        throw FieldError{std::string("missing field ") + key};
    return it->second;
}

std::uint64_t as_u64(const Json& v, const char* key, std::uint64_t max)
{
    if (v.kind != Json::Number || v.text.empty() || v.text[0] == '-' ||
        v.text.find_first_of(".eE") != std::string::npos)
        throw FieldError{std::string(key) + " must be a non-negative integer"};
    errno = 0;
    char* end = nullptr;
    const unsigned long long x = std::strtoull(v.text.c_str(), &end, 10);
    if (errno != 0 || *end != '\0' || x > max)
        throw FieldError{std::string(key) + " is out of range"};
    return x;
}

std::uint64_t get_u64(const Json& o, const char* key)
{
    return as_u64(need(o, key), key, std::numeric_limits<std::uint64_t>::max());
}

std::uint32_t get_u32(const Json& o, const char* key)
{
    return static_cast<std::uint32_t>(
        as_u64(need(o, key), key, std::numeric_limits<std::uint32_t>::max()));
}

double get_double(const Json& o, const char* key)
{
    const Json& v = need(o, key);
    if (v.kind != Json::Number) throw FieldError{std::string(key) + " must be a number"};
    char* end = nullptr;
    const double x = std::strtod(v.text.c_str(), &end);
    if (*end != '\0') throw FieldError{std::string(key) + " is not a number"};
    return x;
}

std::string get_string(const Json& o, const char* key)
{
    const Json& v = need(o, key);
    if (v.kind != Json::String) throw FieldError{std::string(key) + " must be a string"};
    return v.text;
}

bool power_of_two(std::uint64_t v) { return v != 0 && (v & (v - 1)) == 0; }

const char* kSchemes[] = {"CWDP", "CWPD", "CDWP", "CDPW", "CPWD", "CPDW",
                          "WCDP", "WCPD", "WDCP", "WDPC", "WPCD", "WPDC",
                          "DCWP", "DCPW", "DWCP", "DWPC", "DPCW", "DPWC",
                          "PCWD", "PCDW", "PWCD", "PWDC", "PDCW", "PDWC"};

}  // namespace

std::uint64_t channel_bandwidth(const Profile& p)
{
    return static_cast<std::uint64_t>(p.channel_width_bits) *
           p.channel_transfer_rate_mtps * 1000000ull / 8ull;
}

std::string validate_profile(const Profile& p)
{
    if (p.capacity_bytes == 0) return "capacity_bytes must be greater than zero";
    if (!power_of_two(p.page_bytes)) return "page_bytes must be a power of two";
    if (p.page_bytes < 512) return "page_bytes must be at least 512";
    if (p.read_latency_ns == 0) return "read_latency_ns must be greater than zero";
    if (p.program_latency_ns == 0) return "program_latency_ns must be greater than zero";
    if (!p.channels || !p.dies_per_channel || !p.planes_per_die ||
        !p.pages_per_block || !p.channel_width_bits ||
        !p.channel_transfer_rate_mtps || !p.queue_depth)
        return "geometry and channel fields must be greater than zero";
    if (p.aggregate_bandwidth_bytes_per_s == 0)
        return "aggregate_bandwidth_bytes_per_s must be greater than zero";
    if (p.hbm_cache_bytes > p.capacity_bytes)
        return "hbm_cache_bytes must not exceed capacity_bytes";
    if (!std::isfinite(p.reference_sample_rate) || p.reference_sample_rate < 0.0 ||
        p.reference_sample_rate > 1.0)
        return "reference_sample_rate must be in [0, 1]";
    if (p.time_scale == 0) return "time_scale must be greater than zero";
    const unsigned __int128 denominator =
        static_cast<unsigned __int128>(p.page_bytes) * p.channels *
        p.dies_per_channel * p.planes_per_die * p.pages_per_block;
    if (denominator > std::numeric_limits<std::uint64_t>::max() ||
        p.capacity_bytes % static_cast<std::uint64_t>(denominator) != 0 ||
        p.capacity_bytes / static_cast<std::uint64_t>(denominator) == 0)
        return "capacity geometry must contain an integral number of blocks per plane";
    for (auto v : p.page_latency)
        if (v == 0) return "per-level page read/program latencies must be greater than zero";
    bool known = false;
    for (auto s : kSchemes) known = known || p.plane_allocation_scheme == s;
    if (!known) return "plane_allocation_scheme must be one of the 24 orderings";
    if (p.nand_technology != "SLC" && p.nand_technology != "MLC" &&
        p.nand_technology != "TLC" && p.nand_technology != "QLC")
        return "nand_technology must be one of SLC, MLC, TLC, QLC";
    if (!p.has_empirical) return {};
    if (p.page_bytes != 4096) return "empirical_vmem requires page_bytes == 4096";
    for (int i = 0; i < 6; ++i) {
        const auto& pt = p.empirical[i];
        if (i && pt.pages <= p.empirical[i - 1].pages)
            return "empirical_vmem pages must be strictly increasing";
        if (pt.cumulative_ns == 0 ||
            (i && pt.cumulative_ns <= p.empirical[i - 1].cumulative_ns))
            return "empirical_vmem P50 latency must be strictly increasing";
        if (pt.p95_ns < pt.cumulative_ns) return "empirical_vmem P95 latency must not be below P50";
    }
    if (p.empirical[5].pages > 1023) return "empirical_vmem final page must not exceed 1023";
    if (p.empirical_program_p50_ns == 0) return "empirical_vmem program P50 must be greater than zero";
    if (p.empirical_program_p95_ns < p.empirical_program_p50_ns)
        return "empirical_vmem program P95 must not be below P50";
    return {};
}

std::string load_profile(const std::string& path, Profile* out)
{
    std::ifstream in(path);
    if (!in) return "could not open profile: " + path;
    std::stringstream buf;
    buf << in.rdbuf();
    const std::string text = buf.str();
    Json doc;
    Reader reader(text);
    if (!reader.parse(&doc) || doc.kind != Json::Object) return "invalid profile JSON";
    Profile p;
    try {
        p.name = get_string(doc, "name");
        p.capacity_bytes = get_u64(doc, "capacity_bytes");
        p.page_bytes = get_u32(doc, "page_bytes");
        p.read_latency_ns = get_u64(doc, "read_latency_ns");
        p.program_latency_ns = get_u64(doc, "program_latency_ns");
        p.channels = get_u32(doc, "channels");
        p.dies_per_channel = get_u32(doc, "dies_per_channel");
        p.planes_per_die = get_u32(doc, "planes_per_die");
        p.pages_per_block = get_u32(doc, "pages_per_block");
        p.channel_width_bits = get_u32(doc, "channel_width_bits");
        p.channel_transfer_rate_mtps = get_u32(doc, "channel_transfer_rate_mtps");
        p.queue_depth = get_u32(doc, "queue_depth");
        p.aggregate_bandwidth_bytes_per_s = get_u64(doc, "aggregate_bandwidth_bytes_per_s");
        p.hbm_cache_bytes = get_u64(doc, "hbm_cache_bytes");
        p.reference_sample_rate = get_double(doc, "reference_sample_rate");
        p.reference_warmup_requests = get_u32(doc, "reference_warmup_requests");
        p.time_scale = get_u32(doc, "time_scale");
        p.timing_tolerance_ns = get_u64(doc, "timing_tolerance_ns");
        if (doc.fields.count("nand_technology"))
            p.nand_technology = get_string(doc, "nand_technology");
        if (doc.fields.count("plane_allocation_scheme"))
            p.plane_allocation_scheme = get_string(doc, "plane_allocation_scheme");
        static const char* levels[8] = {
            "page_read_latency_lsb_ns", "page_read_latency_csb_ns",
            "page_read_latency_msb_ns", "page_read_latency_tsb_ns",
            "page_program_latency_lsb_ns", "page_program_latency_csb_ns",
            "page_program_latency_msb_ns", "page_program_latency_tsb_ns"};
        for (int i = 0; i < 8; ++i)
            p.page_latency[i] = doc.fields.count(levels[i])
                                    ? get_u64(doc, levels[i])
                                    : (i < 4 ? p.read_latency_ns : p.program_latency_ns);
        const auto emp = doc.fields.find("empirical_vmem");
        if (emp != doc.fields.end()) {
            const Json& e = emp->second;
            const Json& curve = need(e, "read_curve");
            if (curve.kind != Json::Array || curve.items.size() != 6)
                return "empirical_vmem read_curve must contain exactly 6 points";
            p.has_empirical = true;
            for (int i = 0; i < 6; ++i) {
                p.empirical[i].pages = get_u32(curve.items[i], "pages");
                p.empirical[i].cumulative_ns = get_u64(curve.items[i], "cumulative_ns");
                p.empirical[i].p95_ns = get_u64(curve.items[i], "p95_ns");
            }
            p.empirical_program_p50_ns = get_u64(e, "program_p50_ns");
            p.empirical_program_p95_ns = get_u64(e, "program_p95_ns");
            const std::string sha = get_string(e, "source_sha256");
            if (sha.size() != 64 || sha.find_first_not_of("0123456789abcdef") != std::string::npos)
                return "empirical_vmem source_sha256 must be lowercase hexadecimal SHA256";
            if (get_string(e, "source_kind").empty()) return "empirical_vmem source_kind must not be empty";
            if (get_u64(e, "source_capacity_bytes") == 0)
                return "empirical_vmem source_capacity_bytes must be greater than zero";
            if (get_string(e, "quantile") != "p50") return "empirical_vmem quantile must be p50";
            if (get_u32(e, "sample_count") == 0) return "empirical_vmem sample_count must be greater than zero";
        }
    } catch (const FieldError& error) {
        return "invalid profile JSON: " + error.message;
    }
    const std::string problem = validate_profile(p);
    if (!problem.empty()) return problem;
    *out = p;
    return {};
}

}  // namespace hbfb
