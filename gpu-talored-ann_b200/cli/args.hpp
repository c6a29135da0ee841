// Minimal long-option parser for the command-line tools (the reference's tools use
// boost::program_options; this accepts the same spellings: `--name value`, `--name=value`,
// one-letter aliases, and boolean switches).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace cli {

struct Opt {
    std::string name;   // long name
    char alias;         // one-letter alias or 0
    bool is_switch;     // takes no value
    std::string help;
    std::string deflt;  // shown in --help; empty = none
};

class Args {
public:
    Args(std::string tool, std::vector<Opt> opts) : tool_(std::move(tool)), opts_(std::move(opts)) {}

    // Returns false when --help was given (usage printed).
    bool parse(int argc, char** argv)
    {
        for (int i = 1; i < argc; ++i) {
            std::string a = argv[i];
            std::string key, val;
            bool has_val = false;
            if (a.rfind("--", 0) == 0) {
                key = a.substr(2);
                const size_t eq = key.find('=');
                if (eq != std::string::npos) {
                    val = key.substr(eq + 1);
                    key = key.substr(0, eq);
                    has_val = true;
                }
            } else if (a.size() == 2 && a[0] == '-') {
                key = find_alias(a[1]);
            } else {
                throw std::runtime_error("unexpected argument: " + a);
            }
            if (key == "help" || key == "h") {
                usage();
                return false;
            }
            const Opt* o = find(key);
            if (!o) throw std::runtime_error("unknown option --" + key);
            if (o->is_switch) {
                vals_[o->name] = has_val ? val : "1";
                continue;
            }
            if (!has_val) {
                if (i + 1 >= argc) throw std::runtime_error("option --" + o->name + " needs a value");
                val = argv[++i];
            }
            vals_[o->name] = val;
        }
        return true;
    }

    bool has(const std::string& k) const { return vals_.count(k) != 0; }
    std::string str(const std::string& k, const std::string& d = "") const
    {
        auto it = vals_.find(k);
        return it == vals_.end() ? d : it->second;
    }
    std::string required(const std::string& k) const
    {
        if (!has(k)) throw std::runtime_error("the option --" + k + " is required");
        return str(k);
    }
    int64_t i64(const std::string& k, int64_t d) const
    {
        if (!has(k)) return d;
        char* end = nullptr;
        const std::string s = str(k);
        const long long v = std::strtoll(s.c_str(), &end, 10);
        if (end == s.c_str() || *end) throw std::runtime_error("option --" + k + ": not an integer: " + s);
        return v;
    }
    double f64(const std::string& k, double d) const
    {
        if (!has(k)) return d;
        char* end = nullptr;
        const std::string s = str(k);
        const double v = std::strtod(s.c_str(), &end);
        if (end == s.c_str() || *end) throw std::runtime_error("option --" + k + ": not a number: " + s);
        return v;
    }
    bool flag(const std::string& k) const
    {
        if (!has(k)) return false;
        const std::string v = str(k);
        return !(v == "0" || v == "false" || v == "off");
    }

    void usage() const
    {
        std::printf("%s options:\n", tool_.c_str());
        for (const Opt& o : opts_) {
            std::string lhs = "  ";
            lhs += o.alias ? std::string("-") + o.alias + " [ --" + o.name + " ]" : "--" + o.name;
            if (!o.is_switch) lhs += " arg";
            if (!o.deflt.empty()) lhs += " (=" + o.deflt + ")";
            std::printf("%-44s %s\n", lhs.c_str(), o.help.c_str());
        }
    }

private:
    const Opt* find(const std::string& k) const
    {
        for (const Opt& o : opts_)
            if (o.name == k) return &o;
        return nullptr;
    }
    std::string find_alias(char c) const
    {
        if (c == 'h') return "help";
        for (const Opt& o : opts_)
            if (o.alias == c) return o.name;
        throw std::runtime_error(std::string("unknown option -") + c);
    }

    std::string tool_;
    std::vector<Opt> opts_;
    std::map<std::string, std::string> vals_;
};

}  // namespace cli
