// Data-parallel replicas behind the C ABI (no PyTorch): the batch is sharded by image across
// GPUs, each GPU holds a full copy of the weights and runs the whole forward pass on its
// shard, and the only exchange is the gather of the logits. Images never interact (the
// reference's batch-invariance test, tests/vit_test.cu:203-238), so nothing crosses NVLink
// per layer.
//
// Two forms:
//   * one process per GPU (torchrun-style launchers): cuvit_comm_* wraps an NCCL communicator
//     and cuvit_gather_logits gathers every rank's logits to a root rank with grouped
//     point-to-point sends/receives over NVLink;
//   * one process driving several GPUs (a C++ server on one node): cuvit_replicas_* owns one
//     model per device and one host thread per device; logits come back in global image order
//     to host memory or, peer to peer, into one device's buffer.
// NCCL is loaded at run time (dlopen of libnccl.so.2), so the library itself loads on hosts
// without it; only the cuvit_comm_* calls need it.
#include "cuvit_b200.h"
#include "runtime.hpp"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <condition_variable>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

using cuvit::host::fail;

namespace cuvit::replicas {
namespace {

// ---- NCCL, resolved at run time ------------------------------------------------------------

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t,
                         cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

int nccl(const NcclApi** out) {
    static NcclApi api;
    static std::string error;
    static std::once_flag once;
    std::call_once(once, []() {
        void* handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (handle == nullptr) {
            handle = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        }
        if (handle == nullptr) {
            error = "NCCL (libnccl.so.2) cannot be loaded";
            return;
        }
        const auto bind = [&](auto& slot, const char* name) {
            slot = reinterpret_cast<std::remove_reference_t<decltype(slot)>>(dlsym(handle, name));
            if (slot == nullptr && error.empty()) {
                error = std::string("NCCL lacks ") + name;
            }
        };
        bind(api.get_unique_id, "ncclGetUniqueId");
        bind(api.comm_init_rank, "ncclCommInitRank");
        bind(api.comm_destroy, "ncclCommDestroy");
        bind(api.group_start, "ncclGroupStart");
        bind(api.group_end, "ncclGroupEnd");
        bind(api.send, "ncclSend");
        bind(api.recv, "ncclRecv");
        bind(api.error_string, "ncclGetErrorString");
    });
    if (!error.empty()) {
        return fail(CUVIT_UNSUPPORTED, error);
    }
    *out = &api;
    return CUVIT_OK;
}

int check_nccl(const NcclApi& api, ncclResult_t result, const char* what) {
    if (result == ncclSuccess) {
        return CUVIT_OK;
    }
    return fail(CUVIT_RUNTIME_ERROR,
                std::string("NCCL call failed: ") + what + " (" + api.error_string(result) + ")");
}

// ---- a fixed team of host threads, one per device ----------------------------------------

class Team {
  public:
    explicit Team(int members) : members_(members) {
        for (int i = 0; i < members_; ++i) {
            workers_.emplace_back([this, i] { work(i); });
        }
    }
    ~Team() {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            stop_ = true;
        }
        start_.notify_all();
        for (std::thread& worker : workers_) {
            worker.join();
        }
    }
    Team(const Team&) = delete;
    Team& operator=(const Team&) = delete;

    // Runs job(member) on every member's thread and returns the first non-OK status (with
    // that member's message), after all have finished.
    int run(const std::function<int(int)>& job) {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            job_ = &job;
            pending_ = members_;
            statuses_.assign(static_cast<size_t>(members_), CUVIT_OK);
            messages_.assign(static_cast<size_t>(members_), std::string());
            ++generation_;
        }
        start_.notify_all();
        std::unique_lock<std::mutex> lock(mutex_);
        done_.wait(lock, [this] { return pending_ == 0; });
        job_ = nullptr;
        for (int i = 0; i < members_; ++i) {
            if (statuses_[static_cast<size_t>(i)] != CUVIT_OK) {
                return fail(statuses_[static_cast<size_t>(i)],
                            "device " + std::to_string(i) + ": " +
                                messages_[static_cast<size_t>(i)]);
            }
        }
        return CUVIT_OK;
    }

  private:
    void work(int member) {
        uint64_t seen = 0;
        for (;;) {
            const std::function<int(int)>* job = nullptr;
            {
                std::unique_lock<std::mutex> lock(mutex_);
                start_.wait(lock, [&] { return stop_ || generation_ != seen; });
                if (stop_) {
                    return;
                }
                seen = generation_;
                job = job_;
            }
            const int status = (*job)(member);
            const std::string message = status == CUVIT_OK ? "" : cuvit_last_error_message();
            {
                std::lock_guard<std::mutex> lock(mutex_);
                statuses_[static_cast<size_t>(member)] = status;
                messages_[static_cast<size_t>(member)] = message;
                if (--pending_ == 0) {
                    done_.notify_one();
                }
            }
        }
    }

    const int members_;
    std::vector<std::thread> workers_;
    std::mutex mutex_;
    std::condition_variable start_;
    std::condition_variable done_;
    const std::function<int(int)>* job_ = nullptr;
    std::vector<int> statuses_;
    std::vector<std::string> messages_;
    uint64_t generation_ = 0;
    int pending_ = 0;
    bool stop_ = false;
};

} // namespace
} // namespace cuvit::replicas

struct cuvit_comm {
    ncclComm_t comm = nullptr;
    int world = 0;
    int rank = 0;
    int device = 0;
};

struct cuvit_replicas {
    cuvit_vit_config config{};
    std::vector<int> devices;
    std::vector<cuvit_vit*> models;
    std::vector<cudaStream_t> streams;
    std::vector<float*> logits;    // per device: its shard's logits (device memory)
    std::vector<float*> images;    // per device: its shard's images (device memory)
    std::vector<cudaEvent_t> done; // per device: its part of the current call is complete
    int max_batch = 0;             // per device
    std::unique_ptr<cuvit::replicas::Team> team;
};

namespace {

using cuvit::replicas::NcclApi;

class DeviceScope {
  public:
    explicit DeviceScope(int device) {
        cudaGetDevice(&previous_);
        cudaSetDevice(device);
    }
    ~DeviceScope() { cudaSetDevice(previous_); }

  private:
    int previous_ = 0;
};

void release(cuvit_replicas* r) {
    r->team.reset();
    for (size_t i = 0; i < r->devices.size(); ++i) {
        DeviceScope scope(r->devices[i]);
        if (i < r->models.size() && r->models[i] != nullptr) {
            cuvit_vit_destroy(r->models[i]);
        }
        if (i < r->logits.size() && r->logits[i] != nullptr) {
            cudaFree(r->logits[i]);
        }
        if (i < r->images.size() && r->images[i] != nullptr) {
            cudaFree(r->images[i]);
        }
        if (i < r->done.size() && r->done[i] != nullptr) {
            cudaEventDestroy(r->done[i]);
        }
        if (i < r->streams.size() && r->streams[i] != nullptr) {
            cudaStreamDestroy(r->streams[i]);
        }
    }
}

int check_batch(const cuvit_replicas* r, int batch) {
    if (r == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "replicas cannot be null");
    }
    const long long capacity = static_cast<long long>(r->max_batch) * r->devices.size();
    if (batch < 0 || batch > capacity) {
        return fail(CUVIT_INVALID_ARGUMENT,
                    "These replicas hold at most " + std::to_string(capacity) +
                        " images per call, but " + std::to_string(batch) + " were given");
    }
    return CUVIT_OK;
}

} // namespace

extern "C" {

int cuvit_shard(int total, int parts, int index, int* first, int* count) {
    if (first == nullptr || count == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "shard outputs cannot be null");
    }
    if (total < 0 || parts < 1 || index < 0 || index >= parts) {
        return fail(CUVIT_INVALID_ARGUMENT, "shard index outside the partition");
    }
    const int base = total / parts;
    const int extra = total % parts;
    *first = index * base + (index < extra ? index : extra);
    *count = base + (index < extra ? 1 : 0);
    return CUVIT_OK;
}

int cuvit_comm_unique_id(void* id, size_t capacity) {
    if (id == nullptr || capacity < sizeof(ncclUniqueId)) {
        return fail(CUVIT_INVALID_ARGUMENT,
                    "the unique id needs " + std::to_string(sizeof(ncclUniqueId)) + " bytes");
    }
    const NcclApi* api = nullptr;
    CUVIT_TRY(cuvit::replicas::nccl(&api));
    ncclUniqueId unique{};
    CUVIT_TRY(cuvit::replicas::check_nccl(*api, api->get_unique_id(&unique), "ncclGetUniqueId"));
    std::memcpy(id, &unique, sizeof(unique));
    return CUVIT_OK;
}

int cuvit_comm_create(const void* id, int world, int rank, int device, cuvit_comm** comm) {
    if (id == nullptr || comm == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "communicator arguments cannot be null");
    }
    *comm = nullptr;
    if (world < 1 || rank < 0 || rank >= world || device < 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "rank outside the world, or a negative device");
    }
    const NcclApi* api = nullptr;
    CUVIT_TRY(cuvit::replicas::nccl(&api));
    ncclUniqueId unique{};
    std::memcpy(&unique, id, sizeof(unique));
    DeviceScope scope(device);
    auto made = std::make_unique<cuvit_comm>();
    made->world = world;
    made->rank = rank;
    made->device = device;
    CUVIT_TRY(cuvit::replicas::check_nccl(
        *api, api->comm_init_rank(&made->comm, world, unique, rank), "ncclCommInitRank"));
    *comm = made.release();
    return CUVIT_OK;
}

int cuvit_comm_destroy(cuvit_comm* comm) {
    if (comm == nullptr) {
        return CUVIT_OK;
    }
    const NcclApi* api = nullptr;
    int status = cuvit::replicas::nccl(&api);
    if (status == CUVIT_OK && comm->comm != nullptr) {
        DeviceScope scope(comm->device);
        status = cuvit::replicas::check_nccl(*api, api->comm_destroy(comm->comm),
                                             "ncclCommDestroy");
    }
    delete comm;
    return status;
}

int cuvit_gather_logits(cuvit_comm* comm, const float* local, float* gathered, int rows,
                        int classes, int root, cuvit_stream_t stream) {
    if (comm == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "communicator cannot be null");
    }
    if (rows < 0 || classes <= 0 || root < 0 || root >= comm->world) {
        return fail(CUVIT_INVALID_ARGUMENT, "gather extents or root out of range");
    }
    if (rows == 0) {
        return CUVIT_OK;
    }
    if (local == nullptr || (comm->rank == root && gathered == nullptr)) {
        return fail(CUVIT_INVALID_ARGUMENT, "gather buffers cannot be null");
    }
    const NcclApi* api = nullptr;
    CUVIT_TRY(cuvit::replicas::nccl(&api));
    DeviceScope scope(comm->device);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t count = static_cast<size_t>(rows) * classes;
    if (comm->rank == root) {
        // The root's own slice is a device copy; the others arrive in rank order, so the
        // gathered rows are in global image order for contiguous shards.
        CUVIT_TRY_CUDA(cudaMemcpyAsync(gathered + count * root, local, count * sizeof(float),
                                       cudaMemcpyDeviceToDevice, s));
        if (comm->world > 1) {
            CUVIT_TRY(cuvit::replicas::check_nccl(*api, api->group_start(), "ncclGroupStart"));
            for (int peer = 0; peer < comm->world; ++peer) {
                if (peer != root) {
                    const ncclResult_t result = api->recv(gathered + count * peer, count,
                                                          ncclFloat32, peer, comm->comm, s);
                    if (result != ncclSuccess) {
                        api->group_end();
                        return cuvit::replicas::check_nccl(*api, result, "ncclRecv");
                    }
                }
            }
            CUVIT_TRY(cuvit::replicas::check_nccl(*api, api->group_end(), "ncclGroupEnd"));
        }
        return CUVIT_OK;
    }
    CUVIT_TRY(cuvit::replicas::check_nccl(*api, api->group_start(), "ncclGroupStart"));
    const ncclResult_t result = api->send(local, count, ncclFloat32, root, comm->comm, s);
    const ncclResult_t ended = api->group_end();
    CUVIT_TRY(cuvit::replicas::check_nccl(*api, result, "ncclSend"));
    return cuvit::replicas::check_nccl(*api, ended, "ncclGroupEnd");
}

int cuvit_replicas_create(const cuvit_vit_config* config, const float* const* tensors,
                          int tensor_count, int max_batch_per_device, int precision,
                          const int* devices, int device_count, cuvit_replicas** out) {
    if (out == nullptr || config == nullptr || tensors == nullptr || devices == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "replica creation arguments cannot be null");
    }
    *out = nullptr;
    if (device_count < 1) {
        return fail(CUVIT_INVALID_ARGUMENT, "at least one device is needed");
    }
    int available = 0;
    CUVIT_TRY_CUDA(cudaGetDeviceCount(&available));
    for (int i = 0; i < device_count; ++i) {
        if (devices[i] < 0 || devices[i] >= available) {
            return fail(CUVIT_INVALID_ARGUMENT,
                        "device " + std::to_string(devices[i]) + " does not exist");
        }
    }
    auto r = std::make_unique<cuvit_replicas>();
    r->config = *config;
    r->max_batch = max_batch_per_device;
    r->devices.assign(devices, devices + device_count);
    r->models.assign(static_cast<size_t>(device_count), nullptr);
    r->streams.assign(static_cast<size_t>(device_count), nullptr);
    r->logits.assign(static_cast<size_t>(device_count), nullptr);
    r->images.assign(static_cast<size_t>(device_count), nullptr);
    r->done.assign(static_cast<size_t>(device_count), nullptr);
    const size_t image_elements =
        static_cast<size_t>(config->channels) * config->image_size * config->image_size;
    int status = CUVIT_OK;
    for (int i = 0; i < device_count && status == CUVIT_OK; ++i) {
        status = cuvit_vit_create_from_host(config, tensors, tensor_count, max_batch_per_device,
                                            precision, devices[i], &r->models[i]);
        if (status != CUVIT_OK) {
            break;
        }
        DeviceScope scope(devices[i]);
        status = cuvit::host::check_cuda(
            cudaStreamCreateWithFlags(&r->streams[i], cudaStreamNonBlocking),
            "cudaStreamCreateWithFlags");
        if (status == CUVIT_OK) {
            status = cuvit::host::check_cuda(
                cudaEventCreateWithFlags(&r->done[i], cudaEventDisableTiming), "cudaEventCreate");
        }
        if (status == CUVIT_OK) {
            status = cuvit::host::check_cuda(
                cudaMalloc(&r->logits[i], static_cast<size_t>(max_batch_per_device) *
                                              config->classes * sizeof(float)),
                "cudaMalloc(replica logits)");
        }
        if (status == CUVIT_OK) {
            status = cuvit::host::check_cuda(
                cudaMalloc(&r->images[i],
                           static_cast<size_t>(max_batch_per_device) * image_elements *
                               sizeof(float)),
                "cudaMalloc(replica images)");
        }
    }
    if (status != CUVIT_OK) {
        release(r.get());
        return status;
    }
    r->team = std::make_unique<cuvit::replicas::Team>(device_count);
    *out = r.release();
    return CUVIT_OK;
}

int cuvit_replicas_destroy(cuvit_replicas* replicas) {
    if (replicas == nullptr) {
        return CUVIT_OK;
    }
    for (size_t i = 0; i < replicas->devices.size(); ++i) {
        DeviceScope scope(replicas->devices[i]);
        cudaDeviceSynchronize();
    }
    release(replicas);
    delete replicas;
    return CUVIT_OK;
}

int cuvit_replicas_device_count(const cuvit_replicas* replicas) {
    return replicas ? static_cast<int>(replicas->devices.size()) : 0;
}

int cuvit_replicas_forward_host(cuvit_replicas* replicas, const float* images, float* logits,
                                int batch) {
    CUVIT_TRY(check_batch(replicas, batch));
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (images == nullptr || logits == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "Forward pass operands cannot be null");
    }
    cuvit_replicas& r = *replicas;
    const int parts = static_cast<int>(r.devices.size());
    const size_t per_image =
        static_cast<size_t>(r.config.channels) * r.config.image_size * r.config.image_size;
    const size_t classes = static_cast<size_t>(r.config.classes);
    // Each device's thread moves its contiguous shard host -> device, runs the pass and
    // writes its logits straight into the caller's rows: the result is in global order.
    return r.team->run([&](int part) -> int {
        int first = 0;
        int count = 0;
        CUVIT_TRY(cuvit_shard(batch, parts, part, &first, &count));
        if (count == 0) {
            return CUVIT_OK;
        }
        if (count > r.max_batch) {
            return fail(CUVIT_INVALID_ARGUMENT, "shard exceeds the per-device batch");
        }
        return cuvit_vit_forward_host(r.models[part], images + per_image * first,
                                      logits + classes * first, count,
                                      reinterpret_cast<cuvit_stream_t>(r.streams[part]));
    });
}

int cuvit_replicas_forward(cuvit_replicas* replicas, const float* images, int images_device,
                           float* logits, int logits_device, int batch) {
    CUVIT_TRY(check_batch(replicas, batch));
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (images == nullptr || logits == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "Forward pass operands cannot be null");
    }
    cuvit_replicas& r = *replicas;
    const int parts = static_cast<int>(r.devices.size());
    const size_t per_image =
        static_cast<size_t>(r.config.channels) * r.config.image_size * r.config.image_size;
    const size_t classes = static_cast<size_t>(r.config.classes);
    // Each device pulls its shard peer to peer from images_device, replays the pass and pushes
    // its logits peer to peer into logits_device's buffer at its rows.
    return r.team->run([&](int part) -> int {
        int first = 0;
        int count = 0;
        CUVIT_TRY(cuvit_shard(batch, parts, part, &first, &count));
        if (count == 0) {
            return CUVIT_OK;
        }
        if (count > r.max_batch) {
            return fail(CUVIT_INVALID_ARGUMENT, "shard exceeds the per-device batch");
        }
        const int device = r.devices[static_cast<size_t>(part)];
        DeviceScope scope(device);
        const cudaStream_t s = r.streams[static_cast<size_t>(part)];
        CUVIT_TRY_CUDA(cudaMemcpyPeerAsync(r.images[part], device, images + per_image * first,
                                           images_device, per_image * count * sizeof(float), s));
        CUVIT_TRY(cuvit_vit_forward_graph(r.models[part], r.images[part], r.logits[part], count,
                                          reinterpret_cast<cuvit_stream_t>(s)));
        CUVIT_TRY_CUDA(cudaMemcpyPeerAsync(logits + classes * first, logits_device,
                                           r.logits[part], device,
                                           classes * count * sizeof(float), s));
        CUVIT_TRY_CUDA(cudaStreamSynchronize(s));
        return cuvit::host::peek_device_status();
    });
}

} // extern "C"
