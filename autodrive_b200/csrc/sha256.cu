// SHA-256 (FIPS 180-4) of fixed-size chunks, one thread per chunk, with a
// host twin built from the same source. Used for provenance digests of
// checkpoints and playback records: leaf digests of `chunk`-byte slices of a
// byte buffer (the last chunk may be short), and a binary hash tree over them
// (parent = SHA-256(left || right), an odd node is promoted unchanged).
// Reference role: frc_defense/meco_tree_digest_hip.py, csrc/meco_tree_digest_hip_kernel.cu:9.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <vector>

namespace py = pybind11;

namespace {

#if defined(__CUDACC__)
#define SHA_HD __host__ __device__ __forceinline__
#else
#define SHA_HD inline
#endif

// FIPS 180-4 section 4.2.2: first 32 bits of the fractional parts of the cube
// roots of the first 64 primes; section 5.3.3: initial hash value.
#define SHA256_K_TABLE                                                                                      \
  {0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u, \
   0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u, \
   0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, \
   0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u, \
   0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, \
   0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u, \
   0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u, \
   0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u}

__constant__ uint32_t kK_dev[64] = SHA256_K_TABLE;
static const uint32_t kK_host[64] = SHA256_K_TABLE;

SHA_HD uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

SHA_HD void compress(uint32_t* h, const uint32_t* block_words) {
#if defined(__CUDA_ARCH__)
  const uint32_t* K = kK_dev;
#else
  const uint32_t* K = kK_host;
#endif
  uint32_t w[64];
  for (int t = 0; t < 16; ++t) w[t] = block_words[t];
  for (int t = 16; t < 64; ++t) {
    const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = w[t - 16] + s0 + w[t - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int t = 0; t < 64; ++t) {
    const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + K[t] + w[t];
    const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = S0 + maj;
    hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

// Digest of `len` bytes at `msg` into out[32] (big-endian words).
SHA_HD void sha256(const uint8_t* msg, uint64_t len, uint8_t* out) {
  uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  uint32_t blk[16];
  const uint64_t total = ((len + 9 + 63) / 64) * 64;  // padded length
  for (uint64_t off = 0; off < total; off += 64) {
    for (int i = 0; i < 16; ++i) {
      uint32_t word = 0;
      for (int k = 0; k < 4; ++k) {
        const uint64_t p = off + (uint64_t)i * 4 + k;
        uint8_t byte;
        if (p < len) byte = msg[p];
        else if (p == len) byte = 0x80u;
        else if (p >= total - 8) byte = (uint8_t)(((len * 8) >> (8 * (total - 1 - p))) & 0xffu);
        else byte = 0;
        word = (word << 8) | byte;
      }
      blk[i] = word;
    }
    compress(h, blk);
  }
  for (int i = 0; i < 8; ++i)
    for (int k = 0; k < 4; ++k) out[i * 4 + k] = (uint8_t)(h[i] >> (24 - 8 * k));
}

__global__ void sha256_chunks_kernel(const uint8_t* __restrict__ data, uint64_t nbytes, uint64_t chunk,
                                     int64_t nchunks, uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nchunks) return;
  const uint64_t off = (uint64_t)i * chunk;
  const uint64_t len = (off + chunk <= nbytes) ? chunk : nbytes - off;
  sha256(data + off, len, out + i * 32);
}

__global__ void sha256_pairs_kernel(const uint8_t* __restrict__ level, int64_t n, uint8_t* __restrict__ next) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * i + 1 < n) {
    sha256(level + 2 * i * 32, 64, next + i * 32);  // two adjacent 32-byte digests
  } else if (2 * i < n) {
    for (int k = 0; k < 32; ++k) next[i * 32 + k] = level[2 * i * 32 + k];
  }
}

torch::Tensor chunk_digests(torch::Tensor data, int64_t chunk) {
  TORCH_CHECK(chunk > 0, "chunk must be positive");
  auto bytes = data.contiguous().view(torch::kUInt8).reshape({-1});
  const uint64_t n = (uint64_t)bytes.numel();
  const int64_t nchunks = n == 0 ? 1 : (int64_t)((n + chunk - 1) / chunk);
  auto out = torch::empty({nchunks, 32}, bytes.options());
  if (bytes.is_cuda()) {
    auto st = c10::cuda::getCurrentCUDAStream().stream();
    sha256_chunks_kernel<<<(unsigned)((nchunks + 127) / 128), 128, 0, st>>>(bytes.data_ptr<uint8_t>(), n, (uint64_t)chunk,
                                                                           nchunks, out.data_ptr<uint8_t>());
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "sha256_chunks_kernel launch failed");
  } else {
    const uint8_t* d = bytes.data_ptr<uint8_t>();
    uint8_t* o = out.data_ptr<uint8_t>();
    for (int64_t i = 0; i < nchunks; ++i) {
      const uint64_t off = (uint64_t)i * chunk;
      const uint64_t len = (off + chunk <= n) ? chunk : n - off;
      sha256(d + off, len, o + i * 32);
    }
  }
  return out;
}

// Root of the binary hash tree over the chunk digests.
torch::Tensor tree_digest(torch::Tensor data, int64_t chunk) {
  auto level = chunk_digests(data, chunk);
  while (level.size(0) > 1) {
    const int64_t n = level.size(0), m = (n + 1) / 2;
    auto next = torch::empty({m, 32}, level.options());
    if (level.is_cuda()) {
      auto st = c10::cuda::getCurrentCUDAStream().stream();
      sha256_pairs_kernel<<<(unsigned)((m + 127) / 128), 128, 0, st>>>(level.data_ptr<uint8_t>(), n,
                                                                        next.data_ptr<uint8_t>());
      TORCH_CHECK(cudaGetLastError() == cudaSuccess, "sha256_pairs_kernel launch failed");
    } else {
      const uint8_t* l = level.data_ptr<uint8_t>();
      uint8_t* o = next.data_ptr<uint8_t>();
      for (int64_t i = 0; i < m; ++i) {
        if (2 * i + 1 < n) sha256(l + 2 * i * 32, 64, o + i * 32);
        else std::memcpy(o + i * 32, l + 2 * i * 32, 32);
      }
    }
    level = next;
  }
  return level.reshape({32});
}

}  // namespace

void register_sha256_ops(py::module& m) {
  m.def("sha256_chunks", &chunk_digests, "SHA-256 of each `chunk`-byte slice of a tensor's bytes -> [n, 32] uint8",
        py::arg("data"), py::arg("chunk"));
  m.def("sha256_tree", &tree_digest, "root of the binary SHA-256 tree over the chunk digests -> [32] uint8",
        py::arg("data"), py::arg("chunk") = 1 << 16);
}
