// Symmetric heap over NVLink peer memory, plus the two small kernels that
// the fused Ulysses GEMMs need around them.
//
// Every rank of a context-parallel group allocates one device region of the
// same size (cudaMalloc, so it is exportable), exports it with a CUDA IPC
// handle and maps every peer's region into its own address space. Slots
// are carved at identical offsets on every rank (a bump allocator driven by
// the same sequence of calls), so `peer_base[r] + offset` is rank r's copy of
// a slot. The first kSignalBytes of each region are the barrier's signal
// words: word [s] of rank r is written only by rank s.
//
// * heap_barrier: all ranks of the heap meet. Each rank bumps a device-side
//   epoch (so a captured graph replays correctly), stores it into its word
//   of every peer's signal area with a system-scope release, and waits with
//   a system-scope acquire until every peer's word in its own area reached
//   the epoch. The wait is bounded by wall time (globaltimer); on expiry it
//   records kSitePeer in the device error slot and returns.
// * gather_rows: the sequence-layout copy of rank-sharded head buffers,
//   read over NVLink with 16-byte loads (used where a weight gradient needs
//   the gathered activation as a plain local operand).
//
// There is no NVLS object and no multimem access here: every transfer
// is a plain peer load or store.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <vector>

#include "../common/peer.cuh"
#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kMaxRanks = 8;
constexpr int64_t kSignalBytes = 4096;          // signal words; epoch counter at byte 2048

struct SignalPtrs {
  unsigned int* word[kMaxRanks];                // rank r's signal area
};

struct SourcePtrs {
  const uint4* p[kMaxRanks];                    // rank r's slot
};

__global__ void heap_barrier_kernel(SignalPtrs sig, int rank, int world, uint64_t timeout_ns, ErrorSlot* err) {
  __shared__ unsigned int epoch;
  unsigned int* counter = sig.word[rank] + 512;          // local, byte offset 2048
  if (threadIdx.x == 0) epoch = *counter + 1u;
  __syncthreads();
  __threadfence_system();
  const int peer = threadIdx.x;
  if (peer < world) store_release_sys(sig.word[peer] + rank, epoch);
  if (peer < world) {
    const unsigned int* mine = sig.word[rank] + peer;
    const uint64_t start = global_ns();
    while (static_cast<int>(load_acquire_sys(mine) - epoch) < 0) {
      if (global_ns() - start > timeout_ns) {
        report(err, kSitePeer);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = epoch;
}

// dst[b, t, part * dim + owner * C + c] = src_owner[part, b, rank * n_local + t, c]
__global__ void gather_rows_kernel(SourcePtrs src, uint4* dst, int world, int rank, int parts, int batch, int n_local,
                                   int C) {
  const int c16 = C / 8;                                   // 16-byte units per owner row
  const int row_units = parts * world * c16;
  const int64_t total = static_cast<int64_t>(batch) * n_local * row_units;
  const int n_total = n_local * world;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / row_units;
    const int u = static_cast<int>(i - row * row_units);
    const int b = static_cast<int>(row / n_local), t = static_cast<int>(row - static_cast<int64_t>(b) * n_local);
    const int part = u / (world * c16);
    const int rest = u - part * world * c16;
    const int owner = rest / c16, cu = rest - owner * c16;
    dst[i] = src.p[owner][(static_cast<int64_t>(part * batch + b) * n_total + rank * n_local + t) * c16 + cu];
  }
}

}  // namespace

int64_t heap_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  EB_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(bytes)));
  EB_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(bytes)));
  EB_CUDA_CHECK(cudaDeviceSynchronize());
  return reinterpret_cast<int64_t>(ptr);
}

void heap_free(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  EB_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

at::Tensor heap_ipc_handle(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t handle;
  EB_CUDA_CHECK(cudaIpcGetMemHandle(&handle, reinterpret_cast<void*>(ptr)));
  at::Tensor out = at::empty({static_cast<int64_t>(sizeof(handle))}, at::kByte);
  std::memcpy(out.data_ptr(), &handle, sizeof(handle));
  return out;
}

int64_t heap_open(const at::Tensor& handle, int64_t device) {
  TORCH_CHECK(handle.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)), "heap_open: bad handle");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* ptr = nullptr;
  EB_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void heap_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  EB_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// A tensor view of `bytes_offset` into a heap region (no ownership).
at::Tensor heap_tensor(int64_t base, int64_t bytes_offset, at::IntArrayRef sizes, at::ScalarType dtype,
                       int64_t device) {
  auto options = at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  return at::from_blob(reinterpret_cast<char*>(base) + bytes_offset, sizes, options);
}

int64_t heap_signal_bytes() { return kSignalBytes; }

void heap_barrier(const std::vector<int64_t>& bases, int64_t rank, double timeout_s) {
  const int world = static_cast<int>(bases.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "heap_barrier: bad world/rank");
  SignalPtrs sig{};
  for (int r = 0; r < world; ++r) sig.word[r] = reinterpret_cast<unsigned int*>(bases[r]);
  const int device = at::cuda::current_device();
  const uint64_t timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  heap_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(sig, static_cast<int>(rank), world, timeout_ns,
                                                                      device_error_slot(device));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

// Sequence-layout copy [batch * n_local, parts * world * C] of rank-sharded
// head buffers (src[r] = rank r's [parts, batch, n_total, C] slot).
void gather_rows(const std::vector<int64_t>& src, int64_t rank, int64_t parts, int64_t batch, int64_t n_local,
                 int64_t C, at::Tensor& out) {
  const int world = static_cast<int>(src.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && C % 8 == 0, "gather_rows: bad layout");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.scalar_type() == at::kBFloat16 &&
                  out.numel() == batch * n_local * parts * world * C,
              "gather_rows: out must be contiguous bf16 [batch * n_local, parts * world * C]");
  const c10::cuda::CUDAGuard guard(out.device());
  SourcePtrs table{};
  for (int r = 0; r < world; ++r) {
    TORCH_CHECK(src[r] % 16 == 0, "gather_rows: sources must be 16-byte aligned");
    table.p[r] = reinterpret_cast<const uint4*>(src[r]);
  }
  const int64_t units = out.numel() / 8;
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((units + threads - 1) / threads, 148 * 8));
  gather_rows_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      table, reinterpret_cast<uint4*>(out.data_ptr()), world,
      static_cast<int>(rank), static_cast<int>(parts), static_cast<int>(batch), static_cast<int>(n_local),
      static_cast<int>(C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

}  // namespace eb
