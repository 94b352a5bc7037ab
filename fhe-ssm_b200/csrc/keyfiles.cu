// keyfiles.cu -- seeded key part files and the rotation-index contract (the key material path
// between a client that holds the secret and a server that holds none).
//
// Part file "FSSMSKY1" (the reference's format, hpc_gpu_port/seeded_keys.hpp:44-52, written and
// read by writeSeededPart / readSeededPartHeader / expandSeededKeys, :327-420), all integers
// little-endian:
//   char[8] "FSSMSKY1"; u32 version = 1; u32 expander = 1; u32 N; u32 sizeQ; u32 sizeP;
//   u32 numPartQ; u32 numPerPartQ; u32 count; u32 keyTagLen; keyTag bytes;
//   u64 moduli[sizeQ + sizeP]; then per key: u32 automorphism index; u8 seed[32];
//   u64 b[numPartQ][sizeQ + sizeP][N] in evaluation form (canonical residues).
// The a-halves are not stored: the loader re-expands them from the seed with the normative
// expander (keys.cu, on the device).  A file whose chain or digit layout differs from the
// context's is refused, as the reference's loader refuses it (:388-390).  Keys the context
// already holds are kept (the reference's map insert adds only new indices, :404-418).
// Index 0 carries the relinearisation key (this engine's extension: the reference keeps its
// EvalMultKey in a separate serialisation); automorphism indices are odd, so 0 is free.
//
// Rotation-index contract ("fhe-ssm-rot-indices-v1", gpu_real_model.cu:1337-1394): the
// rotation amounts, the bootstrap steps and the automorphism indices 5^s mod 2N (plus the
// conjugation 2N - 1) a server built with this model will look up; a client keygen that mints
// exactly `autoIndices` (fhe_keygen_rotations) serves it.
#include <cstdio>
#include <fstream>
#include <set>

namespace {

constexpr char kPartMagic[8] = {'F', 'S', 'S', 'M', 'S', 'K', 'Y', '1'};
constexpr uint32_t kPartVersion = 1, kPartExpander = 1;

void put32(std::ostream& os, uint32_t v) {
    const uint8_t b[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
    os.write((const char*)b, 4);
}
void put64(std::ostream& os, uint64_t v) {
    uint8_t b[8];
    for (int i = 0; i < 8; i++) b[i] = (uint8_t)(v >> (8 * i));
    os.write((const char*)b, 8);
}
bool get32(std::istream& is, uint32_t& v) {
    uint8_t b[4];
    if (!is.read((char*)b, 4)) return false;
    v = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    return true;
}
bool get64(std::istream& is, uint64_t& v) {
    uint8_t b[8];
    if (!is.read((char*)b, 8)) return false;
    v = 0;
    for (int i = 0; i < 8; i++) v |= (uint64_t)b[i] << (8 * i);
    return true;
}

struct PartHead {
    fhe_part_layout lay{};
    std::vector<uint64_t> moduli;
    std::string tag;
};

void write_head(std::ostream& os, const fhe_part_layout& L, const uint64_t* moduli, const std::string& tag) {
    os.write(kPartMagic, 8);
    put32(os, kPartVersion);
    put32(os, kPartExpander);
    put32(os, L.N); put32(os, L.sizeQ); put32(os, L.sizeP);
    put32(os, L.numPartQ); put32(os, L.numPerPartQ); put32(os, L.count);
    put32(os, (uint32_t)tag.size());
    os.write(tag.data(), (std::streamsize)tag.size());
    for (uint32_t i = 0; i < L.sizeQ + L.sizeP; i++) put64(os, moduli[i]);
}

void read_head(std::istream& is, PartHead& H) {
    char magic[8];
    if (!is.read(magic, 8) || std::memcmp(magic, kPartMagic, 8) != 0) throw fhe::Error("part file: bad magic", FHE_ERR_ARG);
    fhe_part_layout& L = H.lay;
    uint32_t tl = 0;
    const bool ok = get32(is, L.version) && get32(is, L.expander) && get32(is, L.N) && get32(is, L.sizeQ) &&
                    get32(is, L.sizeP) && get32(is, L.numPartQ) && get32(is, L.numPerPartQ) && get32(is, L.count) &&
                    get32(is, tl);
    if (!ok) throw fhe::Error("part file: short header", FHE_ERR_ARG);
    if (L.version != kPartVersion || L.expander != kPartExpander)
        throw fhe::Error("part file: unsupported version/expander", FHE_ERR_ARG);
    if (tl > 4096) throw fhe::Error("part file: keyTag too long", FHE_ERR_ARG);
    if (L.sizeQ + L.sizeP > 256 || L.N > (1u << 17)) throw fhe::Error("part file: implausible layout", FHE_ERR_ARG);
    H.tag.assign(tl, '\0');
    if (tl && !is.read(&H.tag[0], tl)) throw fhe::Error("part file: short keyTag", FHE_ERR_ARG);
    H.moduli.resize(L.sizeQ + L.sizeP);
    for (auto& m : H.moduli)
        if (!get64(is, m)) throw fhe::Error("part file: short moduli", FHE_ERR_ARG);
}

fhe_part_layout context_layout(const fhe::Context& c, uint32_t count) {
    fhe_part_layout L{};
    L.version = kPartVersion; L.expander = kPartExpander;
    L.N = (uint32_t)c.N; L.sizeQ = (uint32_t)c.L; L.sizeP = (uint32_t)c.K;
    L.numPartQ = (uint32_t)c.dnum_top; L.numPerPartQ = (uint32_t)c.alpha; L.count = count;
    return L;
}

}  // namespace

namespace fhe {
// the rotation amounts a model's step uses (BSGS babies and giants, the rmsnorm block sums up and
// down); the conjugation and the bootstrap's steps come on top
std::vector<int> model_rotation_steps(const ModelCfg& cfg);
}

extern "C" {

int fhe_part_header(const char* path, fhe_part_layout* lay, uint64_t* moduli, int moduli_cap, char* tag,
                    int tag_cap) {
    return guard([&] {
        REQUIRE(path && lay, "null argument");
        std::ifstream is(path, std::ios::binary);
        REQUIRE(is.good(), std::string("cannot open ") + path);
        PartHead H;
        read_head(is, H);
        *lay = H.lay;
        if (moduli) {
            REQUIRE((int)H.moduli.size() <= moduli_cap, "moduli buffer too small");
            std::memcpy(moduli, H.moduli.data(), H.moduli.size() * 8);
        }
        if (tag) {
            REQUIRE((int)H.tag.size() < tag_cap, "tag buffer too small");
            std::memcpy(tag, H.tag.c_str(), H.tag.size() + 1);
        }
    });
}

int fhe_part_write_words(const char* path, const fhe_part_layout* lay, const uint64_t* moduli, const char* tag,
                         const uint32_t* indices, const uint8_t* seeds, const uint64_t* b) {
    return guard([&] {
        REQUIRE(path && lay && moduli && tag && (lay->count == 0 || (indices && seeds && b)), "null argument");
        REQUIRE(*tag, "empty key tag");
        std::ofstream os(path, std::ios::binary | std::ios::trunc);
        REQUIRE(os.good(), std::string("cannot open ") + path);
        write_head(os, *lay, moduli, tag);
        const size_t words = (size_t)lay->numPartQ * (lay->sizeQ + lay->sizeP) * lay->N;
        for (uint32_t k = 0; k < lay->count; k++) {
            put32(os, indices[k]);
            os.write((const char*)seeds + 32 * (size_t)k, 32);
            os.write((const char*)(b + k * words), (std::streamsize)(words * 8));   // little-endian hosts
        }
        os.flush();
        REQUIRE(os.good(), std::string("write failed: ") + path);
    });
}

int fhe_keys_save_part(fhe_ctx* cx, const char* path, const uint64_t* which, int n, const char* tag) {
    return guard([&] {
        REQUIRE(cx && path && which && n > 0 && tag && *tag, "bad argument");
        bind(cx);
        auto& c = cx->cx;
        const int nm = c.L + c.K, N = c.N;
        std::vector<fhe::SwitchKey*> keys(n);
        for (int i = 0; i < n; i++) {
            keys[i] = find_key(c, which[i]);
            REQUIRE(keys[i]->seeded, "key " + std::to_string(which[i]) +
                                         " was not generated from a seed; it cannot go into a seeded part file");
        }
        const fhe_part_layout L = context_layout(c, (uint32_t)n);
        std::ofstream os(path, std::ios::binary | std::ios::trunc);
        REQUIRE(os.good(), std::string("cannot open ") + path);
        write_head(os, L, c.mods.data(), tag);
        const size_t words = (size_t)c.dnum_top * nm * N;
        fhe::DevBuf t(words, c.stream);
        std::vector<uint64_t> host(words);
        for (int i = 0; i < n; i++) {
            // the b-halves [digit][limb][N], out of the Montgomery form the key is kept in
            for (int j = 0; j < c.dnum_top; j++)
                CUDA_CHECK(cudaMemcpyAsync(t.p + (size_t)j * nm * N, keys[i]->buf.p + (size_t)j * 2 * nm * N,
                                           (size_t)nm * N * 8, cudaMemcpyDeviceToDevice, c.stream));
            fhe::k_mont<<<dim3(N / 256, c.dnum_top * nm), 256, 0, c.stream>>>(t.p, nm, 0, c.logN);
            CUDA_CHECK(cudaGetLastError());
            c.launches++;
            fhe::download(c, host.data(), t.p, words);
            put32(os, (uint32_t)which[i]);
            os.write((const char*)keys[i]->seed, 32);
            os.write((const char*)host.data(), (std::streamsize)(words * 8));
        }
        os.flush();
        REQUIRE(os.good(), std::string("write failed: ") + path);
    });
}

int fhe_keys_load_part(fhe_ctx* cx, const char* path, int* inserted) {
    return guard([&] {
        REQUIRE(cx && path, "null argument");
        bind(cx);
        auto& c = cx->cx;
        std::ifstream is(path, std::ios::binary);
        REQUIRE(is.good(), std::string("cannot open ") + path);
        PartHead H;
        read_head(is, H);
        const fhe_part_layout L = context_layout(c, H.lay.count);
        const bool same = H.lay.N == L.N && H.lay.sizeQ == L.sizeQ && H.lay.sizeP == L.sizeP &&
                          H.lay.numPartQ == L.numPartQ && H.lay.numPerPartQ == L.numPerPartQ &&
                          H.moduli == c.mods;
        REQUIRE(same, std::string("part file ") + path + " was minted for another context (N/chain/digits differ)");
        REQUIRE(!H.tag.empty(), "empty keyTag");
        const int nm = c.L + c.K, N = c.N;
        const size_t words = (size_t)c.dnum_top * nm * N;
        std::vector<uint64_t> bw(words);
        int added = 0;
        for (uint32_t r = 0; r < H.lay.count; r++) {
            uint32_t index = 0;
            uint8_t seed[32];
            if (!get32(is, index) || !is.read((char*)seed, 32) || !is.read((char*)bw.data(), (std::streamsize)(words * 8)))
                throw fhe::Error("short key record " + std::to_string(r) + " in " + path, FHE_ERR_ARG);
            REQUIRE(index == 0 || (index & 1), "key record " + std::to_string(r) + ": even automorphism index");
            REQUIRE(index < 2ull * N, "key record " + std::to_string(r) + ": automorphism index out of range");
            if (index == 0 ? (bool)c.rlk : c.rot_keys.count(index) > 0) continue;
            auto key = std::make_unique<fhe::SwitchKey>();
            key->buf = fhe::DevBuf((size_t)c.dnum_top * 2 * nm * N, c.stream);
            key->index = index;
            std::memcpy(key->seed, seed, 32);
            key->seeded = true;
            for (int j = 0; j < c.dnum_top; j++)
                CUDA_CHECK(cudaMemcpyAsync(key->buf.p + (size_t)j * 2 * nm * N, bw.data() + (size_t)j * nm * N,
                                           (size_t)nm * N * 8, cudaMemcpyHostToDevice, c.stream));
            fhe::expand_uniform_dev(c, seed, 0, c.dnum_top, 0, nm, fhe::kTagSKEY, key->buf.p + (size_t)nm * N,
                                    (long long)2 * nm * N);
            fhe::k_mont<<<dim3(N / 256, c.dnum_top * 2 * nm), 256, 0, c.stream>>>(key->buf.p, nm, 1, c.logN);
            CUDA_CHECK(cudaGetLastError());
            c.launches++;
            CUDA_CHECK(cudaStreamSynchronize(c.stream));   // bw is reused for the next record
            c.check_device_error();
            if (index == 0) c.rlk = std::move(key);
            else c.rot_keys[index] = std::move(key);
            added++;
        }
        if (inserted) *inserted = added;
    });
}

int fhe_model_rot_contract(const fhe_model* m, char* buf, int cap) {
    return guard([&] {
        REQUIRE(m && buf && cap > 2, "null argument");
        const auto& c = m->owner->cx;
        const auto& cfg = m->m->cfg;
        std::vector<int> rots = fhe::model_rotation_steps(cfg);
        std::sort(rots.begin(), rots.end());
        rots.erase(std::unique(rots.begin(), rots.end()), rots.end());
        std::vector<int> boot;
        if (c.prm.boot_primes > 0) boot = fhe::boot_rotations(c);
        std::set<uint64_t> need;
        for (int s : rots) if (s) need.insert(fhe::rot_index(c, s));
        for (int s : boot) if (s) need.insert(fhe::rot_index(c, s));
        need.insert(2ull * c.N - 1);
        need.erase(1);
        auto arr = [](const auto& v) {
            std::string o = "[";
            bool first = true;
            for (auto x : v) { o += (first ? "" : ",") + std::to_string(x); first = false; }
            return o + "]";
        };
        const std::string js = "{\"contract\":\"fhe-ssm-rot-indices-v1\",\"ring\":" + std::to_string(c.N) +
                               ",\"slots\":" + std::to_string(c.N / 2) + ",\"dpad\":" + std::to_string(cfg.D) +
                               ",\"bs\":" + std::to_string(cfg.b1) + ",\"numDigits\":" + std::to_string(c.dnum_top) +
                               ",\"rotationAmounts\":" + arr(rots) + ",\"bootstrapSteps\":" + arr(boot) +
                               ",\"autoIndices\":" + arr(need) + "}";
        REQUIRE((int)js.size() < cap, "buffer too small");
        std::memcpy(buf, js.c_str(), js.size() + 1);
    });
}

}  // extern "C"
