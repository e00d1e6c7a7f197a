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
#include <functional>
#include <queue>
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

    // BpeTokenizer.Encode (BpeTokenizer.cs:259-318).  Its result is defined
    // as rank-greedy merging: while some adjacent pair has a merge rank,
    // merge the pair of lowest rank, its leftmost occurrence first.
    //
    // This implementation keeps the byte positions as nodes of a list (a node
    // stands for the token that starts at its position) and a min-heap of
    // candidate merges ordered by (rank, position).  A heap entry records the
    // version of its left node; a node's version changes whenever its token
    // or its right neighbour changes, so an entry whose pair no longer exists
    // is recognised and dropped when it surfaces.  Popping (rank, position)
    // in order is the rank-greedy rule: a merge only creates pairs that
    // contain its new id, and such a pair has a higher rank than the merge
    // that made the id (Load requires merges to reference earlier ids).
    std::vector<int32_t> encode(const uint8_t* data, size_t n) const {
        std::vector<int32_t> out;
        if (n == 0) return out;
        struct Node {
            int32_t token;
            int32_t right;    // next live node, -1 at the end
            int32_t left;     // previous live node, -1 at the start
            uint32_t version;
        };
        struct Cand {
            int32_t rank, pos;
            uint32_t version;
            bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
        };
        std::vector<Node> nodes(n);
        for (size_t i = 0; i < n; i++)
            nodes[i] = Node{data[i], i + 1 < n ? (int32_t)(i + 1) : -1, (int32_t)i - 1, 0u};
        std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
        auto offer = [&](int32_t pos) {  // the pair starting at live node pos, if it merges
            const int32_t r = nodes[(size_t)pos].right;
            if (r < 0) return;
            auto it = rank.find(key(nodes[(size_t)pos].token, nodes[(size_t)r].token));
            if (it != rank.end()) heap.push(Cand{it->second, pos, nodes[(size_t)pos].version});
        };
        for (size_t i = 0; i + 1 < n; i++) offer((int32_t)i);
        while (!heap.empty()) {
            const Cand c = heap.top();
            heap.pop();
            Node& a = nodes[(size_t)c.pos];
            if (a.version != c.version) continue;  // pair changed since it was offered
            Node& b = nodes[(size_t)a.right];
            a.token = 256 + c.rank;
            a.right = b.right;
            a.version++;
            if (b.right >= 0) nodes[(size_t)b.right].left = c.pos;
            b.version++;  // b is absorbed; its entries are stale now
            if (a.left >= 0) {
                nodes[(size_t)a.left].version++;  // its right neighbour's token changed
                offer(a.left);
            }
            offer(c.pos);
        }
        for (int32_t i = 0; i >= 0; i = nodes[(size_t)i].right) out.push_back(nodes[(size_t)i].token);
        return out;
    }
};

}  // namespace tok
}  // namespace fb2
