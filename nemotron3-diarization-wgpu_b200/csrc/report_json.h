// JSON text as serde_json writes it, for the `diarize` report (src/bin/diarize.rs
// prints its report with serde_json): numbers in ryu's shortest round-trip form and
// layout, strings with serde_json's escapes.  Host only.
#pragma once

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace n3d {
namespace report {

// The shortest decimal digit string that reads back as v (finite, > 0), with v =
// digits x 10^exp: the correctly rounded p-digit form for the smallest p that
// round-trips.
inline void shortest_digits(double v, std::string& digits, int& exp) {
    char buf[40];
    for (int p = 1; p <= 17; p++) {
        std::snprintf(buf, sizeof buf, "%.*e", p - 1, v);
        if (std::strtod(buf, nullptr) == v) break;
    }
    const char* e = std::strchr(buf, 'e');
    digits.clear();
    for (const char* c = buf; c < e; c++)
        if (*c >= '0' && *c <= '9') digits += *c;
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    exp = std::atoi(e + 1) - (int)(digits.size() - 1);
}

// A JSON number as serde_json prints an f64.  With kk the decimal exponent of the
// leading digit plus one:
// * integral values below 1e16 end in ".0";
// * values with -5 < kk <= 16 are plain decimals;
// * everything else is d.ddd e kk-1, with no '+' and no leading zeros in the exponent.
// Non-finite values become null.
inline std::string number(double v) {
    if (!std::isfinite(v)) return "null";
    std::string out = std::signbit(v) ? "-" : "";
    v = std::fabs(v);
    if (v == 0.0) return out + "0.0";
    std::string d;
    int e = 0;
    shortest_digits(v, d, e);
    const int len = (int)d.size(), kk = len + e;
    if (e >= 0 && kk <= 16) {  // 1234e7 -> 12340000000.0
        out += d;
        out.append((size_t)e, '0');
        out += ".0";
    } else if (kk > 0 && kk <= 16) {  // 1234e-2 -> 12.34
        out += d.substr(0, (size_t)kk) + "." + d.substr((size_t)kk);
    } else if (kk > -5 && kk <= 0) {  // 1234e-6 -> 0.001234
        out += "0.";
        out.append((size_t)-kk, '0');
        out += d;
    } else if (len == 1) {  // 1e30
        out += d + "e" + std::to_string(kk - 1);
    } else {  // 1234e30 -> 1.234e33
        out += d.substr(0, 1) + "." + d.substr(1) + "e" + std::to_string(kk - 1);
    }
    return out;
}

// A JSON string as serde_json escapes it: quote and backslash, the short escapes
// \b \t \n \f \r, and \u00xx (lower-case hex) for the other control characters.
inline std::string quote(const std::string& s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        switch (c) {
            case '"': o += "\\\""; break;
            case '\\': o += "\\\\"; break;
            case '\b': o += "\\b"; break;
            case '\t': o += "\\t"; break;
            case '\n': o += "\\n"; break;
            case '\f': o += "\\f"; break;
            case '\r': o += "\\r"; break;
            default:
                if (c < 0x20) {
                    char u[8];
                    std::snprintf(u, sizeof u, "\\u%04x", c);
                    o += u;
                } else {
                    o += (char)c;
                }
        }
    }
    return o + "\"";
}

}  // namespace report
}  // namespace n3d
