// Byte-level BPE tokenizer (src/LLM.Core/Tokenizer/BpeTokenizer.cs), host side.
//
// Ids 0..255 are the raw bytes; merge k (rank k) makes id 256 + k from the
// ids (left, right); the end-of-sequence token follows the merges and stands
// for no bytes.  The file is the JSON BpeTokenizer.Save writes
// (BpeTokenizer.cs:341-351): {"Version": 2, "Merges": [[left, right, id],
// ...], "EosTokenId": n}, validated as BpeTokenizer.Load does
// (BpeTokenizer.cs:353-389).
#pragma once
#include <cstdint>
#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "forgemodel.hpp"

namespace fb2 {
namespace tok {

struct Bpe {
    std::vector<std::vector<uint8_t>> vocab;  // id -> bytes
    std::vector<int> left, right;             // per rank
    std::unordered_map<uint64_t, int> rank;   // (left, right) -> rank
    int eos = -1;

    static uint64_t key(int l, int r) { return ((uint64_t)(uint32_t)l << 32) | (uint32_t)r; }

    static Bpe load(const char* path) {
        std::vector<unsigned char> bytes;
        {
            std::unique_ptr<FILE, int (*)(FILE*)> fp(std::fopen(path, "rb"), std::fclose);
            if (!fp) throw std::runtime_error(std::string("cannot open '") + path + "'");
            unsigned char buf[1 << 16];
            size_t n;
            while ((n = std::fread(buf, 1, sizeof buf, fp.get())) > 0) bytes.insert(bytes.end(), buf, buf + n);
        }
        fm::Json j;
        try {
            size_t at = 0;
            if (bytes.size() >= 3 && bytes[0] == 0xEF && bytes[1] == 0xBB && bytes[2] == 0xBF) at = 3;  // UTF-8 BOM
            j = fm::JsonParser(reinterpret_cast<const char*>(bytes.data() + at), bytes.size() - at).parse();
        } catch (const std::runtime_error&) {
            throw fm::InvalidData("tokenizer file is empty or malformed");
        }
        if (j.kind != fm::Json::Obj) throw fm::InvalidData("tokenizer file is empty or malformed");
        const fm::Json* ver = j.get("Version");
        const long long v = ver && ver->kind == fm::Json::Num && ver->is_int ? ver->inum : 0;
        if (v != 2) throw fm::InvalidData("unsupported tokenizer version " + std::to_string(v));
        Bpe t;
        for (int i = 0; i < 256; i++) t.vocab.push_back({(uint8_t)i});
        const fm::Json* merges = j.get("Merges");
        if (merges && merges->kind == fm::Json::Arr) {
            for (size_t i = 0; i < merges->arr.size(); i++) {
                const fm::Json& m = merges->arr[i];
                if (m.kind != fm::Json::Arr || m.arr.size() != 3)
                    throw fm::InvalidData("merge " + std::to_string(i) + " must have exactly 3 entries");
                long long e[3];
                for (int k = 0; k < 3; k++) {
                    if (m.arr[k].kind != fm::Json::Num || !m.arr[k].is_int)
                        throw fm::InvalidData("merge " + std::to_string(i) + " entries must be integers");
                    e[k] = m.arr[k].inum;
                }
                const long long n = (long long)t.vocab.size();
                if (e[0] < 0 || e[0] >= n || e[1] < 0 || e[1] >= n)
                    throw fm::InvalidData("merge " + std::to_string(i) + " references unknown token ids");
                if (e[2] != n)
                    throw fm::InvalidData("merge " + std::to_string(i) + " has id " + std::to_string(e[2]) + ", expected " +
                                          std::to_string(n) + " (ids must be 256 + rank)");
                std::vector<uint8_t> b = t.vocab[(size_t)e[0]];
                b.insert(b.end(), t.vocab[(size_t)e[1]].begin(), t.vocab[(size_t)e[1]].end());
                t.vocab.push_back(std::move(b));
                t.left.push_back((int)e[0]);
                t.right.push_back((int)e[1]);
                t.rank[key((int)e[0], (int)e[1])] = (int)i;
            }
        } else if (merges && merges->kind != fm::Json::Null) {
            throw fm::InvalidData("tokenizer file is empty or malformed");
        }
        const fm::Json* eos = j.get("EosTokenId");
        const long long ev = eos && eos->kind == fm::Json::Num && eos->is_int ? eos->inum : 0;
        if (ev != (long long)t.vocab.size())
            throw fm::InvalidData("EOS token has id " + std::to_string(ev) + ", expected " + std::to_string(t.vocab.size()));
        t.eos = (int)t.vocab.size();
        t.vocab.push_back({});
        return t;
    }

    // BpeTokenizer.Encode (BpeTokenizer.cs:259-318): ranks in learned order;
    // per rank a queue of positions whose pair had that rank when enqueued,
    // merged in queue order if still current; merges enqueue the new
    // neighbouring pairs at their (later) ranks.
    std::vector<int32_t> encode(const uint8_t* data, size_t n) const {
        std::vector<int32_t> out;
        if (n == 0) return out;
        std::vector<int> seq(n), next(n), prev(n);
        for (size_t i = 0; i < n; i++) {
            seq[i] = data[i];
            next[i] = i + 1 < n ? (int)i + 1 : -1;
            prev[i] = (int)i - 1;
        }
        std::vector<std::deque<int>> queues(left.size());
        auto rank_of = [&](int a, int b) {
            auto it = rank.find(key(a, b));
            return it == rank.end() ? -1 : it->second;
        };
        for (size_t i = 0; i + 1 < n; i++) {
            const int r = rank_of(seq[i], seq[i + 1]);
            if (r >= 0) queues[(size_t)r].push_back((int)i);
        }
        for (size_t r = 0; r < queues.size(); r++) {
            std::deque<int>& q = queues[r];
            const int new_id = 256 + (int)r;
            while (!q.empty()) {
                const int i = q.front();
                q.pop_front();
                const int j = next[(size_t)i];
                if (j < 0) continue;
                if (rank_of(seq[(size_t)i], seq[(size_t)j]) != (int)r) continue;  // stale
                seq[(size_t)i] = new_id;
                const int nj = next[(size_t)j];
                next[(size_t)i] = nj;
                next[(size_t)j] = -1;
                prev[(size_t)j] = -1;
                if (nj >= 0) {
                    prev[(size_t)nj] = i;
                    const int r2 = rank_of(new_id, seq[(size_t)nj]);
                    if (r2 >= 0) queues[(size_t)r2].push_back(i);
                }
                const int p = prev[(size_t)i];
                if (p >= 0) {
                    const int r3 = rank_of(seq[(size_t)p], new_id);
                    if (r3 >= 0) queues[(size_t)r3].push_back(p);
                }
            }
        }
        for (int i = 0; i >= 0; i = next[(size_t)i]) out.push_back(seq[(size_t)i]);
        return out;
    }
};

}  // namespace tok
}  // namespace fb2
