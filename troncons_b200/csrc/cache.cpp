// troncons_b200 — the expert cache of the streaming path (trc-cache, moteur/crates/trc-cache):
// two tiers, device slots for experts and host entries ("tiedes") for their coded parts, an LRU
// or Belady replacement order per tier, the pinning of a layer's experts, the slot state machine
// (Libre -> EnVol -> Present -> Libre on eviction), the counters, the routing-trace reader and the
// replay that runs a trace through the same code (trc-cache/src/lib.rs:105-301,
// politiques.rs:1-260, trace.rs:1-171).
//
// Rules kept from the reference, in its order (lib.rs:136-206): every expert of a request is
// pinned before the first is served; a device miss takes a free slot or evicts the policy's
// victim among the slots neither pinned nor in flight; the host tier is inclusive and sees every
// access (a device hit also touches the expert's host entry), and a host entry is created only
// by a read from storage; `evictions` counts device evictions. A request whose miss finds no
// free or evictable slot, and `pret` on a slot not in flight, are errors (the reference panics):
// the call returns TRC_ERR_USAGE and the cache must not be used further.
#include <cctype>
#include <cstdarg>
#include <cstdint>
#include <cstdlib>
#include <functional>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/troncons_b200.h"

namespace tb {
int erreur_usage(const char* message);
}

namespace {

using Id = uint32_t;  // couche << 16 | expert: the order of (couche, expert) pairs
constexpr uint32_t NUL = 0xFFFFFFFFu;

inline Id id_de(uint16_t couche, uint16_t expert) { return (uint32_t(couche) << 16) | expert; }

int usage(const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    return tb::erreur_usage(b);
}

// A replacement order over the identifiers present in one tier (politiques.rs:13-23): told of
// each hit (acceder), entry (inserer) and exit (retirer); `victime` names the one to evict among
// those the predicate does not protect, without removing it.
struct Politique {
    virtual ~Politique() = default;
    virtual void acceder(Id id, uint64_t t) = 0;
    virtual void inserer(Id id, uint64_t t) = 0;
    virtual void retirer(Id id) = 0;
    virtual bool victime(const std::function<bool(Id)>& protege, Id& v) = 0;
};

// LRU (politiques.rs:47-160): a doubly linked list in arrays, oldest at the head; a hit moves
// the identifier to the tail; the victim is the oldest not protected.
struct Lru final : Politique {
    struct Noeud {
        Id id;
        uint32_t prec, suiv;
    };
    std::vector<Noeud> noeuds;
    std::vector<uint32_t> libres;
    std::unordered_map<Id, uint32_t> index;
    uint32_t tete = NUL, queue = NUL;

    void detacher(uint32_t i) {
        const Noeud n = noeuds[i];
        if (n.prec == NUL) tete = n.suiv; else noeuds[n.prec].suiv = n.suiv;
        if (n.suiv == NUL) queue = n.prec; else noeuds[n.suiv].prec = n.prec;
    }
    void accrocher_en_queue(uint32_t i) {
        noeuds[i].prec = queue;
        noeuds[i].suiv = NUL;
        if (queue == NUL) tete = i; else noeuds[queue].suiv = i;
        queue = i;
    }
    void acceder(Id id, uint64_t) override {
        const uint32_t i = index.at(id);
        if (i != queue) {
            detacher(i);
            accrocher_en_queue(i);
        }
    }
    void inserer(Id id, uint64_t) override {
        uint32_t i;
        if (!libres.empty()) {
            i = libres.back();
            libres.pop_back();
            noeuds[i] = {id, NUL, NUL};
        } else {
            noeuds.push_back({id, NUL, NUL});
            i = uint32_t(noeuds.size() - 1);
        }
        index[id] = i;
        accrocher_en_queue(i);
    }
    void retirer(Id id) override {
        auto it = index.find(id);
        const uint32_t i = it->second;
        index.erase(it);
        detacher(i);
        libres.push_back(i);
    }
    bool victime(const std::function<bool(Id)>& protege, Id& v) override {
        for (uint32_t i = tete; i != NUL; i = noeuds[i].suiv)
            if (!protege(noeuds[i].id)) {
                v = noeuds[i].id;
                return true;
            }
        return false;
    }
};

// Belady (politiques.rs:162-260): evicts the present, unprotected identifier whose next use is
// furthest; ties (same next group, or never again) go to the smallest (couche, expert). Instants
// are group indices t = token * L + layer, the replay's convention; it reads the future from the
// trace, so it serves the replay only.
struct Belady final : Politique {
    std::unordered_map<Id, std::vector<uint64_t>> usages;
    std::vector<Id> presents;
    std::unordered_map<Id, size_t> rang;
    std::unordered_map<Id, uint64_t> prochain;

    Belady(const uint16_t* choix, uint32_t jetons, uint16_t couches, uint16_t k) {
        for (uint32_t t = 0; t < jetons; ++t)
            for (uint32_t c = 0; c < couches; ++c) {
                const uint64_t instant = uint64_t(t) * couches + c;
                for (uint32_t i = 0; i < k; ++i) {
                    auto& v = usages[id_de(uint16_t(c), choix[(uint64_t(t) * couches + c) * k + i])];
                    if (v.empty() || v.back() != instant) v.push_back(instant);
                }
            }
    }
    // The first use of `id` strictly after t (UINT64_MAX when none): computed at each access,
    // as politiques.rs:208-224 settles it (a present identifier not pinned has not been served
    // since its last access).
    uint64_t prochain_apres(Id id, uint64_t t) const {
        auto it = usages.find(id);
        if (it == usages.end()) return UINT64_MAX;
        const auto& v = it->second;
        size_t lo = 0, hi = v.size();
        while (lo < hi) {
            const size_t m = (lo + hi) / 2;
            if (v[m] <= t) lo = m + 1; else hi = m;
        }
        return lo < v.size() ? v[lo] : UINT64_MAX;
    }
    void acceder(Id id, uint64_t t) override { prochain[id] = prochain_apres(id, t); }
    void inserer(Id id, uint64_t t) override {
        rang[id] = presents.size();
        presents.push_back(id);
        prochain[id] = prochain_apres(id, t);
    }
    void retirer(Id id) override {
        auto it = rang.find(id);
        const size_t i = it->second;
        rang.erase(it);
        presents[i] = presents.back();
        presents.pop_back();
        if (i < presents.size()) rang[presents[i]] = i;
        prochain.erase(id);
    }
    bool victime(const std::function<bool(Id)>& protege, Id& v) override {
        bool trouve = false;
        uint64_t bp = 0;
        Id bid = 0;
        for (Id id : presents) {
            if (protege(id)) continue;
            const uint64_t p = prochain[id];
            if (!trouve || p > bp || (p == bp && id < bid)) {
                trouve = true;
                bp = p;
                bid = id;
            }
        }
        if (trouve) v = bid;
        return trouve;
    }
};

enum EtatEmpl : uint32_t { LIBRE = 0, EN_VOL = 1, PRESENT = 2 };
constexpr uint32_t NIVEAU_EXACT = 1;  // Niveau::Exact (lib.rs:56-60); Base is not used here

}  // namespace

struct trc_cache {
    Politique* vram = nullptr;
    Politique* ram = nullptr;
    bool casser = false;  // the broken policy of the reference's witness: hits are not told
    std::vector<uint32_t> etats, niveaux;
    std::vector<int64_t> occupant;  // Id or -1
    std::unordered_map<Id, uint32_t> ou_vram;
    std::vector<uint32_t> libres_vram;
    std::vector<int64_t> occupant_tiede;
    std::unordered_map<Id, uint32_t> ou_ram;
    std::vector<uint32_t> libres_ram;
    std::vector<Id> epingles;
    std::vector<uint64_t> tailles;  // [couche * experts + expert], empty: bytes are not counted
    uint32_t tailles_experts = 0;
    trc_compteurs_cache compteurs{};

    ~trc_cache() {
        delete vram;
        delete ram;
    }
    bool epingle(Id id) const {
        for (Id e : epingles)
            if (e == id) return true;
        return false;
    }
    uint64_t taille(Id id) const {
        if (tailles.empty()) return 0;
        const uint64_t i = uint64_t(id >> 16) * tailles_experts + (id & 0xFFFFu);
        return i < tailles.size() ? tailles[i] : 0;
    }
    void acceder(Politique* p, Id id, uint64_t t) {
        if (!casser) p->acceder(id, t);
    }

    // A free slot, or the device victim's (evicted here). NUL when none.
    uint32_t emplacement_pour_defaut() {
        if (!libres_vram.empty()) {
            const uint32_t s = libres_vram.back();
            libres_vram.pop_back();
            return s;
        }
        Id v;
        const bool ok = vram->victime(
            [&](Id id) {
                if (epingle(id)) return true;
                auto it = ou_vram.find(id);
                return it != ou_vram.end() && etats[it->second] == EN_VOL;
            },
            v);
        if (!ok) return NUL;
        vram->retirer(v);
        auto it = ou_vram.find(v);
        const uint32_t s = it->second;
        ou_vram.erase(it);
        occupant[s] = -1;
        etats[s] = LIBRE;
        compteurs.evictions += 1;
        return s;
    }

    // A host entry for a part read from storage; -1 without host tier, or when every entry is
    // pinned (the part then goes through an arrival buffer and is not kept).
    int32_t entree_tiede_pour(Id id, uint64_t t) {
        if (occupant_tiede.empty()) return -1;
        uint32_t r;
        if (!libres_ram.empty()) {
            r = libres_ram.back();
            libres_ram.pop_back();
        } else {
            Id v;
            if (!ram->victime([&](Id x) { return epingle(x); }, v)) return -1;
            ram->retirer(v);
            auto it = ou_ram.find(v);
            r = it->second;
            ou_ram.erase(it);
            occupant_tiede[r] = -1;
            compteurs.evictions_ram += 1;
        }
        ram->inserer(id, t);
        occupant_tiede[r] = int64_t(id);
        ou_ram[id] = r;
        return int32_t(r);
    }
};

namespace {

Politique* politique_de(uint32_t p, const uint16_t* choix, uint32_t jetons, uint16_t couches, uint16_t k) {
    if (p == TRC_POLITIQUE_LRU) return new Lru();
    if (p == TRC_POLITIQUE_BELADY && choix != nullptr) return new Belady(choix, jetons, couches, k);
    return nullptr;
}

bool valider_trace(const uint16_t* choix, uint32_t jetons, uint16_t couches, uint16_t k) {
    return choix != nullptr && jetons > 0 && couches > 0 && k > 0;
}

}  // namespace

extern "C" {

trc_cache* trc_cache_nouveau(uint32_t emplacements, uint32_t tiedes, uint32_t politique, const uint16_t* choix,
                             uint32_t jetons, uint16_t couches, uint16_t k, uint32_t casser) {
    if (politique == TRC_POLITIQUE_BELADY && !valider_trace(choix, jetons, couches, k)) {
        usage("Belady needs the trace it replays");
        return nullptr;
    }
    if (politique != TRC_POLITIQUE_LRU && politique != TRC_POLITIQUE_BELADY) {
        usage("policy %u (LRU 0, Belady 1)", politique);
        return nullptr;
    }
    auto* c = new trc_cache();
    c->vram = politique_de(politique, choix, jetons, couches, k);
    c->ram = politique_de(politique, choix, jetons, couches, k);
    c->casser = casser != 0;
    c->etats.assign(emplacements, LIBRE);
    c->niveaux.assign(emplacements, 0);
    c->occupant.assign(emplacements, -1);
    c->ou_vram.reserve(emplacements);
    for (uint32_t s = emplacements; s-- > 0;) c->libres_vram.push_back(s);  // served 0, 1, 2, ...
    c->occupant_tiede.assign(tiedes, -1);
    c->ou_ram.reserve(tiedes);
    for (uint32_t r = tiedes; r-- > 0;) c->libres_ram.push_back(r);
    return c;
}

void trc_cache_detruire(trc_cache* c) { delete c; }

int trc_cache_fixer_tailles(trc_cache* c, const uint64_t* tailles, uint16_t couches, uint16_t experts) {
    if (c == nullptr || tailles == nullptr || couches == 0 || experts == 0) return usage("sizes: a table [couches][experts]");
    c->tailles.assign(tailles, tailles + size_t(couches) * experts);
    c->tailles_experts = experts;
    return TRC_OK;
}

int trc_cache_demander(trc_cache* c, uint16_t couche, const uint16_t* experts, uint32_t n, uint64_t t,
                       trc_decision* decisions) {
    if (c == nullptr || (n > 0 && (experts == nullptr || decisions == nullptr))) return usage("cache request: a buffer is missing");
    for (uint32_t i = 0; i < n; ++i) {
        const Id id = id_de(couche, experts[i]);
        if (!c->epingle(id)) c->epingles.push_back(id);
    }
    for (uint32_t i = 0; i < n; ++i) {
        const Id id = id_de(couche, experts[i]);
        auto it = c->ou_vram.find(id);
        if (it != c->ou_vram.end()) {
            c->acceder(c->vram, id, t);
            if (c->ou_ram.count(id)) c->acceder(c->ram, id, t);
            c->compteurs.succes_vram += 1;
            decisions[i] = {TRC_DECISION_SUCCES, it->second, -1, 0};
            continue;
        }
        const uint32_t s = c->emplacement_pour_defaut();
        if (s == NUL)
            return usage("cache: no free or evictable device slot (%zu slots, %zu experts pinned): slots must be at "
                         "least the experts pinned at once",
                         c->etats.size(), c->epingles.size());
        c->vram->inserer(id, t);
        c->etats[s] = EN_VOL;
        c->niveaux[s] = NIVEAU_EXACT;
        c->occupant[s] = int64_t(id);
        c->ou_vram[id] = s;
        const uint64_t octets = c->taille(id);
        c->compteurs.octets_copies += octets;
        auto r = c->ou_ram.find(id);
        if (r != c->ou_ram.end()) {
            c->acceder(c->ram, id, t);
            c->compteurs.succes_ram += 1;
            decisions[i] = {TRC_DECISION_DEFAUT_RAM, s, int32_t(r->second), 0};
        } else {
            c->compteurs.defauts_disque += 1;
            c->compteurs.octets_disque += octets;
            const int32_t tiede = c->entree_tiede_pour(id, t);
            decisions[i] = {TRC_DECISION_DEFAUT_DISQUE, s, tiede, 0};
        }
    }
    return TRC_OK;
}

int trc_cache_pret(trc_cache* c, uint32_t emplacement) {
    if (c == nullptr || emplacement >= c->etats.size()) return usage("cache: slot %u out of range", emplacement);
    if (c->etats[emplacement] != EN_VOL)
        return usage("cache: ready(%u) on a slot that is %s", emplacement, c->etats[emplacement] == LIBRE ? "free" : "present");
    c->etats[emplacement] = PRESENT;
    return TRC_OK;
}

int trc_cache_liberer(trc_cache* c, uint16_t couche) {
    if (c == nullptr) return usage("cache absent");
    size_t w = 0;
    for (Id id : c->epingles)
        if ((id >> 16) != couche) c->epingles[w++] = id;
    c->epingles.resize(w);
    return TRC_OK;
}

void trc_cache_compteurs(const trc_cache* c, trc_compteurs_cache* sortie) {
    if (c != nullptr && sortie != nullptr) *sortie = c->compteurs;
}

int trc_cache_etat(const trc_cache* c, uint32_t emplacement, uint32_t* etat, uint32_t* niveau) {
    if (c == nullptr || emplacement >= c->etats.size() || etat == nullptr) return usage("cache: slot %u out of range", emplacement);
    *etat = c->etats[emplacement];
    if (niveau != nullptr) *niveau = c->etats[emplacement] == LIBRE ? 0 : c->niveaux[emplacement];
    return TRC_OK;
}

int64_t trc_cache_occupant(const trc_cache* c, uint32_t emplacement) {
    if (c == nullptr || emplacement >= c->occupant.size()) return -1;
    return c->occupant[emplacement];
}

int64_t trc_cache_emplacement_de(const trc_cache* c, uint16_t couche, uint16_t expert) {
    if (c == nullptr) return -1;
    auto it = c->ou_vram.find(id_de(couche, expert));
    return it == c->ou_vram.end() ? -1 : int64_t(it->second);
}

int64_t trc_cache_tiede_de(const trc_cache* c, uint16_t couche, uint16_t expert) {
    if (c == nullptr) return -1;
    auto it = c->ou_ram.find(id_de(couche, expert));
    return it == c->ou_ram.end() ? -1 : int64_t(it->second);
}

uint32_t trc_cache_epingles(const trc_cache* c, uint32_t* ids, uint32_t capacite) {
    if (c == nullptr) return 0;
    const uint32_t n = uint32_t(c->epingles.size());
    for (uint32_t i = 0; i < n && i < capacite && ids != nullptr; ++i) ids[i] = c->epingles[i];
    return n;
}

// The replay (lib.rs:272-301): for each token, each layer in order, request its group at
// t = token * L + layer, mark every miss ready, release the layer.
int trc_rejouer(const uint16_t* choix, uint32_t jetons, uint16_t couches, uint16_t k, uint32_t emplacements,
                uint32_t tiedes, uint32_t politique, uint32_t casser, trc_compteurs_cache* sortie) {
    if (!valider_trace(choix, jetons, couches, k) || sortie == nullptr) return usage("replay: trace or output absent");
    if (emplacements < k) return usage("replay: %u slots < k = %u: a layer would not fit", emplacements, k);
    trc_cache* c = trc_cache_nouveau(emplacements, tiedes, politique, choix, jetons, couches, k, casser);
    if (c == nullptr) return TRC_ERR_USAGE;
    std::vector<trc_decision> d(k);
    int r = TRC_OK;
    for (uint32_t t = 0; t < jetons && r == TRC_OK; ++t)
        for (uint32_t l = 0; l < couches && r == TRC_OK; ++l) {
            r = trc_cache_demander(c, uint16_t(l), choix + (uint64_t(t) * couches + l) * k, k, uint64_t(t) * couches + l,
                                   d.data());
            for (uint32_t i = 0; i < k && r == TRC_OK; ++i)
                if (d[i].sorte != TRC_DECISION_SUCCES) r = trc_cache_pret(c, d[i].emplacement);
            if (r == TRC_OK) trc_cache_liberer(c, uint16_t(l));
        }
    if (r == TRC_OK) *sortie = c->compteurs;
    delete c;
    return r;
}

// ---------------------------------------------------------------- routing traces (trace.rs)

// Reads a trace's text (the format of the reference's tracer): one token per line, layers
// separated by '|', a layer's experts by blanks; '#' lines are comments; "E=<n>" declares the
// experts per layer (else E = largest id + 1). Refused, with the faulty line: a line whose layer
// count differs from the first's, a layer without k experts, an unreadable id, E = 0, an id out
// of [0, E), and an empty trace. `choix` (may be NULL) receives T * L * k ids when `capacite`
// allows; `dims` always receives E, L, k, T, or the error.
int trc_trace_lire(const char* texte, size_t n, trc_trace_dims* dims, uint16_t* choix, size_t capacite) {
    if (dims == nullptr || (texte == nullptr && n > 0)) return usage("trace: dims absent");
    std::memset(dims, 0, sizeof *dims);
    auto erreur = [&](uint32_t sorte, uint32_t numero, const char* raison) {
        dims->erreur = sorte;
        dims->erreur_ligne = numero;
        return usage("trace, line %u: %s", numero, raison);
    };
    int64_t e_declare = -1;
    std::vector<uint16_t> ids;
    uint32_t couches = 0, k = 0, jetons = 0;
    size_t p = 0;
    uint32_t numero = 0;
    while (p < n) {
        size_t q = p;
        while (q < n && texte[q] != '\n') ++q;
        std::string ligne(texte + p, q - p);
        p = q + 1;
        ++numero;
        // trim (Rust str::trim: Unicode white space; the tracer writes ASCII)
        size_t a = 0, b = ligne.size();
        while (a < b && std::isspace(static_cast<unsigned char>(ligne[a]))) ++a;
        while (b > a && std::isspace(static_cast<unsigned char>(ligne[b - 1]))) --b;
        ligne = ligne.substr(a, b - a);
        if (ligne.empty() || ligne[0] == '#') continue;
        if (ligne.rfind("E=", 0) == 0) {
            std::string v = ligne.substr(2);
            size_t x = 0, y = v.size();
            while (x < y && std::isspace(static_cast<unsigned char>(v[x]))) ++x;
            while (y > x && std::isspace(static_cast<unsigned char>(v[y - 1]))) --y;
            v = v.substr(x, y - x);
            char* fin = nullptr;
            const unsigned long e = v.empty() ? 0 : std::strtoul(v.c_str(), &fin, 10);
            // u16::from_str: an optional '+', decimal digits only, at most 65,535
            if (v.empty() || *fin != '\0' || e > 65535 || v[0] == '-' || std::isspace(static_cast<unsigned char>(v[0])) ||
                (v[0] == '+' && v.size() == 1))
                return erreur(1, numero, "unreadable E=");
            if (e == 0) return erreur(1, numero, "E = 0");
            e_declare = int64_t(e);
            continue;
        }
        uint32_t n_couches = 0;
        size_t debut = 0;
        while (true) {
            const size_t barre = ligne.find('|', debut);
            const std::string part = ligne.substr(debut, barre == std::string::npos ? std::string::npos : barre - debut);
            const size_t avant = ids.size();
            size_t i = 0;
            while (i < part.size()) {
                while (i < part.size() && std::isspace(static_cast<unsigned char>(part[i]))) ++i;
                if (i >= part.size()) break;
                size_t j = i;
                while (j < part.size() && !std::isspace(static_cast<unsigned char>(part[j]))) ++j;
                const std::string mot = part.substr(i, j - i);
                char* fin = nullptr;
                const unsigned long x = std::strtoul(mot.c_str(), &fin, 10);
                if (*fin != '\0' || mot[0] == '-' || x > 65535 || (mot[0] == '+' && mot.size() == 1))
                    return erreur(1, numero, "unreadable expert id");
                ids.push_back(uint16_t(x));
                i = j;
            }
            const uint32_t n_couche = uint32_t(ids.size() - avant);
            if (jetons == 0 && n_couches == 0) {
                k = n_couche;
                if (k == 0) return erreur(1, numero, "empty layer");
            } else if (n_couche != k) {
                return erreur(1, numero, "a layer without k experts");
            }
            ++n_couches;
            if (barre == std::string::npos) break;
            debut = barre + 1;
        }
        if (jetons == 0)
            couches = n_couches;
        else if (n_couches != couches)
            return erreur(1, numero, "a line with another layer count than the first");
        ++jetons;
    }
    if (jetons == 0) return erreur(3, 0, "empty trace (no token line)");
    uint16_t max = 0;
    for (uint16_t x : ids) max = x > max ? x : max;
    uint32_t experts;
    if (e_declare >= 0) {
        if (max >= e_declare) {
            dims->erreur = 2;
            dims->erreur_expert = max;
            dims->experts = uint32_t(e_declare);
            return usage("trace: expert %u out of [0, %lld)", max, static_cast<long long>(e_declare));
        }
        experts = uint32_t(e_declare);
    } else {
        experts = uint32_t(max) + 1u;
        if (experts > 65535) {
            dims->erreur = 2;
            dims->erreur_expert = max;
            return usage("trace: expert %u out of range", max);
        }
    }
    dims->experts = experts;
    dims->couches = couches;
    dims->k = k;
    dims->jetons = jetons;
    if (choix != nullptr && capacite >= ids.size()) std::memcpy(choix, ids.data(), ids.size() * sizeof(uint16_t));
    return TRC_OK;
}

}  // extern "C"
