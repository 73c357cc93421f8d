// Host-side check of the ZeRO owner-map arithmetic that the exchange, Adam and owner-scatter kernels run on the GPU
// (csrc/common/zero_map.cuh is __host__ __device__): prints, for sampled flat indices, the owner, the local index,
// the flat index the kernels compute back from (owner, local), and the owner-scatter destination address for
// fake, widely spaced staging bases. tests/test_zero_map_native.py compares them with the Python owner map.
//   zero_map_check <world> <seg> <chunk> <rank> <x0> <count> <stride>
#include <cstdio>
#include <cstdlib>

#include "common/zero_map.cuh"

int main(int argc, char** argv) {
  if (argc != 8) {
    std::fprintf(stderr, "usage: %s world seg chunk rank x0 count stride\n", argv[0]);
    return 2;
  }
  const int world = std::atoi(argv[1]);
  const long long seg = std::atoll(argv[2]), chunk = std::atoll(argv[3]);
  const int rank = std::atoi(argv[4]);
  const long long x0 = std::atoll(argv[5]), count = std::atoll(argv[6]), stride = std::atoll(argv[7]);
  unsigned long long bases[8];
  for (int q = 0; q < 8; ++q) bases[q] = (static_cast<unsigned long long>(q) + 1ull) << 40;   // fake staging bases
  fyb::OwnerScatter sc;
  sc.bases = bases;
  sc.own = reinterpret_cast<__nv_bfloat16*>(static_cast<unsigned long long>(15) << 40);
  sc.x0 = 0;
  sc.seg = seg;
  sc.chunk = chunk;
  sc.rank = rank;
  sc.world = world;
  for (long long i = 0; i < count; ++i) {
    const long long x = x0 + i * stride;
    const int o = fyb::zero_owner(chunk, world, seg, x);
    const long long loc = fyb::zero_local(chunk, world, seg, x);
    const fyb::ZeroMap z{chunk, world, o};
    const long long back = fyb::zero_flat(z, loc) + (chunk == 0 ? static_cast<long long>(o) * seg : 0);
    const unsigned long long dst = reinterpret_cast<unsigned long long>(fyb::owner_dst(sc, x));
    std::printf("%lld %d %lld %lld %llu\n", x, o, loc, back, dst);
  }
  return 0;
}
