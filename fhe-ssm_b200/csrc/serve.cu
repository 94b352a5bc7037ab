// serve.cu -- the stateful serve loop of the reference's server (gpu_real_model.cu:4363-4483,
// driven by ml-eval/fhe_client.py:1394-1493) over the engine's server step.
//
// Protocol, all inside one request directory:
//   client: writes req.<N>.0 .. req.<N>.<count-1> (ciphertexts) and req.<N>.meta (JSON with
//           at least "count"; the reference's other fields are checked when present -- ringDim
//           and level against the ciphertexts, interleave 0, packTokens <= 1 -- and lanes,
//           tokensReal, dpad, packTokens are echoed in resp.<N>.meta), optionally req.<N>.reset
//           (drop the carried state first: a new session), then creates req.<N>.ready.
//   server: runs one step per request in order N = 0, 1, ..., writes resp.<N>.<i>,
//           resp.<N>.meta, then resp.<N>.done -- or resp.<N>.error with the message -- and
//           removes the request files.  serve.status ({"nextReq", "served", "pid",
//           "stateful"}) is rewritten atomically before every wait, so a client that starts
//           against a live server adopts its request counter.
//   exit:   a file named `stop`, or timeout_ms without a request, or max_requests served.
// A malformed request (missing or bad meta, unreadable ciphertext) is answered with
// resp.<N>.error and skipped; the loop never dies on a client's mistake.
//
// Ciphertext files ("FSSMCT01"): magic, int32 level, int32 limbs, int32 logN, int32 pad,
// double scale, then [2][limbs][N] little-endian uint64 residues in evaluation form.  (The
// reference exchanges OpenFHE's cereal serialisation; this engine's files carry the same
// content in raw words.)
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <fstream>
#include <sstream>
#include <thread>

namespace {

bool file_exists(const std::string& p) { return access(p.c_str(), F_OK) == 0; }

void write_text_atomic(const std::string& path, const std::string& body) {
    const std::string tmp = path + ".tmp";
    {
        std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
        f << body;
    }
    std::rename(tmp.c_str(), path.c_str());
}

bool read_text(const std::string& path, std::string& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::stringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

// integer field of a flat JSON object ({"count": 1, "lanes": 64, ...}); false if absent
bool json_int(const std::string& js, const char* key, long long& v) {
    const std::string k = std::string("\"") + key + "\"";
    size_t p = js.find(k);
    if (p == std::string::npos) return false;
    p = js.find(':', p + k.size());
    if (p == std::string::npos) return false;
    p++;
    while (p < js.size() && (js[p] == ' ' || js[p] == '\t')) p++;
    char* end = nullptr;
    v = std::strtoll(js.c_str() + p, &end, 10);
    return end != js.c_str() + p;
}

struct CtFile {
    int level = 0, nl = 0, logN = 0;
    double scale = 0;
    std::vector<uint64_t> words;
};
constexpr char kCtMagic[8] = {'F', 'S', 'S', 'M', 'C', 'T', '0', '1'};

bool read_ct(const std::string& path, CtFile& c) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    char mg[8];
    int32_t h[4];
    f.read(mg, 8);
    f.read(reinterpret_cast<char*>(h), sizeof h);
    f.read(reinterpret_cast<char*>(&c.scale), sizeof c.scale);
    if (!f || std::memcmp(mg, kCtMagic, 8) != 0) return false;
    c.level = h[0]; c.nl = h[1]; c.logN = h[2];
    if (c.nl < 1 || c.nl > 64 || c.logN < 10 || c.logN > 17) return false;
    c.words.resize((size_t)2 * c.nl << c.logN);
    f.read(reinterpret_cast<char*>(c.words.data()), c.words.size() * 8);
    return (bool)f;
}

void write_ct(const std::string& path, const fhe_wire_ct& c) {
    const std::string tmp = path + ".tmp";
    {
        std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
        const int32_t h[4] = {c.level, c.nl, c.logN, 0};
        f.write(kCtMagic, 8);
        f.write(reinterpret_cast<const char*>(h), sizeof h);
        f.write(reinterpret_cast<const char*>(&c.scale), sizeof c.scale);
        f.write(reinterpret_cast<const char*>(c.words), ((size_t)2 * c.nl << c.logN) * 8);
    }
    std::rename(tmp.c_str(), path.c_str());
}

}  // namespace

extern "C" {

int fhe_serve_files(const char* dir, int timeout_ms, int max_requests, fhe_serve_step_fn step, void* user,
                    int* served_out) {
    return guard([&] {
        REQUIRE(dir && step, "null argument");
        const std::string d(dir);
        int N = 0, served = 0;
        const auto idle_ms = [](std::chrono::steady_clock::time_point t0) {
            return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        };
        for (;;) {
            write_text_atomic(d + "/serve.status", "{\"nextReq\":" + std::to_string(N) + ",\"served\":" +
                                                       std::to_string(served) + ",\"pid\":" +
                                                       std::to_string((long long)getpid()) + ",\"stateful\":true}\n");
            if (max_requests > 0 && served >= max_requests) break;
            const std::string req = d + "/req." + std::to_string(N), resp = d + "/resp." + std::to_string(N);
            bool got = false;
            const auto t0 = std::chrono::steady_clock::now();
            for (;;) {
                if (file_exists(d + "/stop")) break;
                if (file_exists(req + ".ready")) { got = true; break; }
                if (timeout_ms >= 0 && idle_ms(t0) > timeout_ms) break;
                std::this_thread::sleep_for(std::chrono::milliseconds(10));
            }
            if (!got) break;
            auto fail = [&](const std::string& why) {
                write_text_atomic(resp + ".error", why + "\n");
                std::remove((req + ".ready").c_str());
                N++;
            };
            std::string meta;
            long long count = -1, mv = 0;
            if (!read_text(req + ".meta", meta) || !json_int(meta, "count", count) || count < 1 || count > 1024) {
                fail("bad or missing request meta");
                continue;
            }
            // the reference's packing fields (gpu_real_model.cu:2333-2340): this engine serves the
            // block layout with one token per lane, so an interleaved or multi-token pack is refused
            if ((json_int(meta, "interleave", mv) && mv != 0) || (json_int(meta, "packTokens", mv) && mv > 1)) {
                fail("request meta asks for an interleaved or multi-token pack; this server runs the block layout");
                continue;
            }
            const bool reset = file_exists(req + ".reset");
            std::vector<CtFile> ins((size_t)count);
            bool ok = true;
            for (long long i = 0; i < count && ok; i++) ok = read_ct(req + "." + std::to_string(i), ins[i]);
            if (!ok) {
                fail("unreadable request ciphertext");
                continue;
            }
            long long ring = 0, lvl = 0;
            for (long long i = 0; i < count && ok; i++)
                ok = (!json_int(meta, "ringDim", ring) || ring == (1LL << ins[i].logN)) &&
                     (!json_int(meta, "level", lvl) || lvl == ins[i].level);
            if (!ok) {
                fail("request meta (ringDim / level) does not match its ciphertexts");
                continue;
            }
            std::vector<fhe_wire_ct> win((size_t)count), wout((size_t)count);
            std::vector<std::vector<uint64_t>> obuf((size_t)count);
            for (long long i = 0; i < count; i++) {
                win[i] = fhe_wire_ct{ins[i].level, ins[i].nl, ins[i].logN, ins[i].scale, ins[i].words.data()};
                obuf[i].assign(ins[i].words.size(), 0);   // an output never has more limbs than its input
                wout[i] = fhe_wire_ct{0, 0, ins[i].logN, 0.0, obuf[i].data()};
            }
            int n_out = 0;
            const int rc = step(user, reset ? 1 : 0, (int)count, win.data(), &n_out, wout.data());
            if (rc != 0 || n_out < 1 || n_out > count) {
                fail(rc != 0 ? std::string("step failed: ") + fhe_last_error() : "step returned no output");
                continue;
            }
            // an output must fit the buffer of its input: same ring, 1..in.nl limbs
            for (int i = 0; i < n_out && ok; i++)
                ok = wout[i].nl >= 1 && wout[i].nl <= ins[i].nl && wout[i].logN == ins[i].logN;
            if (!ok) {
                fail("step returned an output larger than its input or of another ring");
                continue;
            }
            for (int i = 0; i < n_out; i++) write_ct(resp + "." + std::to_string(i), wout[i]);
            // the reference's response meta fields, in its order (writeCtMeta, gpu_real_model.cu:2333-2340)
            long long lanes = 1, toks = 0, pack = 1, dpad = 0;
            json_int(meta, "lanes", lanes);
            json_int(meta, "tokensReal", toks);
            json_int(meta, "packTokens", pack);
            json_int(meta, "dpad", dpad);
            std::string rm = "{\"count\":" + std::to_string(n_out) + ",\"packTokens\":" + std::to_string(pack) +
                             ",\"tokensReal\":" + std::to_string(toks) + ",\"dpad\":" + std::to_string(dpad) +
                             ",\"interleave\":0,\"lanes\":" + std::to_string(lanes) +
                             ",\"ringDim\":" + std::to_string(1LL << wout[0].logN) +
                             ",\"level\":" + std::to_string(wout[0].level) + ",\"reset\":" + (reset ? "true" : "false") + "}\n";
            write_text_atomic(resp + ".meta", rm);
            write_text_atomic(resp + ".done", "ok\n");
            for (long long i = 0; i < count; i++) std::remove((req + "." + std::to_string(i)).c_str());
            std::remove((req + ".meta").c_str());
            std::remove((req + ".reset").c_str());
            std::remove((req + ".ready").c_str());
            served++;
            N++;
        }
        if (served_out) *served_out = served;
    });
}

// the engine's step as a serve callback: user = the fhe_model
static int model_serve_step(void* user, int reset, int n_in, const fhe_wire_ct* in, int* n_out, fhe_wire_ct* out) {
    auto* m = static_cast<fhe_model*>(user);
    fhe_ctx* cx = m->owner;
    if (n_in != 1) {
        g_err = "serve: one input pack per request";
        return FHE_ERR_PROTO;
    }
    if (in[0].logN != cx->cx.logN) {
        g_err = "serve: ring dimension of the request differs from the model's context";
        return FHE_ERR_PROTO;
    }
    fhe_ct* ci = nullptr;
    int rc = fhe_ct_import(cx, in[0].words, in[0].level, in[0].scale, &ci);
    if (rc) return rc;
    fhe_ct* co = nullptr;
    int no = 0;
    rc = fhe_server_step(m, &ci, 1, &co, &no, reset ? 1 : 0);
    fhe_ct_free(ci);
    if (rc) return rc;
    const int nl = co->c.nl;
    if (nl > in[0].nl) {
        fhe_ct_free(co);
        g_err = "serve: output has more limbs than the request";
        return FHE_ERR_PROTO;
    }
    out[0].level = cx->cx.L - nl;
    out[0].nl = nl;
    out[0].logN = cx->cx.logN;
    out[0].scale = co->c.scale;
    rc = fhe_ct_export(cx, co, out[0].words);
    fhe_ct_free(co);
    *n_out = 1;
    return rc;
}

int fhe_serve_model(fhe_model* m, const char* dir, int timeout_ms, int max_requests, int* served) {
    if (!m) {
        g_err = "null argument";
        return FHE_ERR_ARG;
    }
    return fhe_serve_files(dir, timeout_ms, max_requests, model_serve_step, m, served);
}

}  // extern "C"
