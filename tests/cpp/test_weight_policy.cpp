// Driver for tests/test_weight_policy.py: evaluates the weight-precision policy
// of sam.cpp_b200/host/weight_policy.hpp.  Commands, one per line on stdin,
// answers one line each on stdout ("ERROR <message>" on a rejection):
//   sha256 <text with \n escapes>            -> hex digest
//   modules <csv>                            -> parsed list
//   image <profile> <name> <d0> [d1 ...]     -> expected GGML type
//   modular <profile> <modules csv> <name> <d0> [d1 ...]
//   mixed <base> <module csv> <sha> <tensor csv or -> <storage profile or -> <name> <d0> [d1 ...]
//   inspect <gguf path> <expected tensor count>
//                                            -> "<schema> <precision> <modules csv or ->" then one
//                                               "<name> <type>" line per tensor and "END"
#include <iostream>
#include <sstream>

#include "weight_policy.hpp"

using namespace sam::internal::samq_policy;

namespace {

std::string unescape(const std::string& s) {
    std::string out;
    for (std::size_t i = 0; i < s.size(); ++i) {
        if (s[i] == '\\' && i + 1 < s.size() && s[i + 1] == 'n') {
            out.push_back('\n');
            ++i;
        } else {
            out.push_back(s[i]);
        }
    }
    return out;
}

std::vector<std::int64_t> dims_from(std::istringstream& in) {
    std::vector<std::int64_t> dims;
    std::int64_t d;
    while (in >> d) dims.push_back(d);
    return dims;
}

std::string dash(const std::string& s) { return s == "-" ? std::string() : s; }

void run(const std::string& line) {
    std::istringstream in(line);
    std::string cmd;
    in >> cmd;
    if (cmd == "sha256") {
        std::string rest;
        std::getline(in, rest);
        if (!rest.empty() && rest[0] == ' ') rest.erase(0, 1);
        std::cout << sha256_hex(unescape(rest)) << "\n";
    } else if (cmd == "modules") {
        std::string csv;
        in >> csv;
        std::string out;
        for (const auto& m : parse_modules(csv)) out += (out.empty() ? "" : ",") + m;
        std::cout << out << "\n";
    } else if (cmd == "image") {
        std::string profile, name;
        in >> profile >> name;
        const ImageProfile* p = image_profile(profile);
        if (!p) throw std::runtime_error("unsupported SAM GGUF quantization profile");
        std::cout << image_tensor_type(name, dims_from(in), *p) << "\n";
    } else if (cmd == "modular") {
        std::string profile, modules, name;
        in >> profile >> modules >> name;
        const ModularProfile* p = modular_profile(profile);
        if (!p) throw std::runtime_error("unsupported modular SAM GGUF quantization profile");
        std::cout << modular_tensor_type(name, dims_from(in), *p, parse_modules(modules)) << "\n";
    } else if (cmd == "mixed") {
        std::string base, csv, sha, tensors, storage, name;
        in >> base >> csv >> sha >> tensors >> storage >> name;
        const MixedPolicy policy = parse_mixed_policy(base, csv, sha, dash(tensors), dash(storage));
        std::cout << mixed_tensor_type(name, dims_from(in), policy) << "\n";
    } else if (cmd == "inspect") {
        std::string path;
        std::size_t count = 0;
        in >> path >> count;
        GgufReader reader(path);
        const WeightPolicy policy = inspect_weight_policy(reader, count);
        std::string modules;
        for (const auto& m : policy.quantization_modules) modules += (modules.empty() ? "" : ",") + m;
        std::cout << policy.schema << " " << policy.precision << " " << (modules.empty() ? "-" : modules) << "\n";
        for (const auto& t : reader.tensors()) std::cout << t.name << " " << t.type << "\n";
        std::cout << "END\n";
    } else {
        throw std::runtime_error("unknown command " + cmd);
    }
}

}  // namespace

int main() {
    std::string line;
    while (std::getline(std::cin, line)) {
        if (line.empty()) continue;
        try {
            run(line);
        } catch (const std::exception& e) {
            std::cout << "ERROR " << e.what() << "\n";
        }
        std::cout.flush();
    }
    return 0;
}
