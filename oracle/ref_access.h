// ref_access.h -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// engine_of(TemperatureSampler&): the sampler's private std::mt19937 gen_
// (src/sampling/sampling.h:92, seeded from std::random_device in
// sampling.cpp:114-122), so that a test can seed it. Access uses the
// explicit-instantiation access rule ([temp.explicit]/12: access checking
// does not apply to names used in an explicit instantiation), which is
// standard C++ and leaves the class layout untouched.
#pragma once

#include <random>

#include "sampling.h"

namespace qwref_access {

template <typename Tag>
struct MemberPtr {
    static typename Tag::type value;
};
template <typename Tag>
typename Tag::type MemberPtr<Tag>::value;

template <typename Tag, typename Tag::type P>
struct StoreMemberPtr {
    struct Filler {
        Filler() { MemberPtr<Tag>::value = P; }
    };
    static Filler filler;
};
template <typename Tag, typename Tag::type P>
typename StoreMemberPtr<Tag, P>::Filler StoreMemberPtr<Tag, P>::filler;

struct GenTag {
    typedef std::mt19937 qwenium::TemperatureSampler::*type;
};
template struct StoreMemberPtr<GenTag, &qwenium::TemperatureSampler::gen_>;

inline std::mt19937& engine_of(qwenium::TemperatureSampler& s) { return s.*(MemberPtr<GenTag>::value); }

}  // namespace qwref_access
