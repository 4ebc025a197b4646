# rusteeze_b200 serving image for NVIDIA B200 (sm_100a).
#
#   docker build -t rusteeze-b200 .
#   docker run --gpus all --ipc=host -p 8000:8000 -v $PWD/models:/models:ro \
#       rusteeze-b200 serve --model /models/Meta-Llama-3-8B-Instruct --tensor-parallel-size 8
#
# The default command serves with /app/config.yaml (RUSTEEZE_CONFIG; the image
# ships config.example.yaml there, a mounted file replaces it).
#
# Stage 1 compiles the two native extensions in-tree (the CUDA kernels for
# sm_100a only, the C++ host runtime) against the image's PyTorch; stage 2
# carries the package and the built .so files onto a runtime base.  nvcc
# cross-compiles, so the build stage needs no GPU.  --ipc=host (or a large
# --shm-size) is required for tensor parallelism: ranks exchange their step
# plans through a POSIX shared-memory ring and CUDA IPC handles.

ARG CUDA_VERSION=12.9.1
ARG UBUNTU=ubuntu24.04

FROM nvidia/cuda:${CUDA_VERSION}-devel-${UBUNTU} AS build
ENV DEBIAN_FRONTEND=noninteractive PIP_NO_CACHE_DIR=1 VIRTUAL_ENV=/opt/venv PATH=/opt/venv/bin:$PATH
RUN apt-get update && apt-get install -y --no-install-recommends python3 python3-venv python3-dev git ninja-build \
    && rm -rf /var/lib/apt/lists/* && python3 -m venv /opt/venv
COPY requirements.txt /tmp/requirements.txt
RUN pip install --upgrade pip wheel setuptools pybind11 && pip install -r /tmp/requirements.txt
WORKDIR /src
COPY setup.py __graft_entry__.py ./
COPY rusteeze_b200 ./rusteeze_b200
RUN MAX_JOBS=8 python setup.py build_ext --inplace && python -c "import rusteeze_b200._host"

FROM nvidia/cuda:${CUDA_VERSION}-runtime-${UBUNTU} AS runtime
ENV DEBIAN_FRONTEND=noninteractive VIRTUAL_ENV=/opt/venv PATH=/opt/venv/bin:$PATH PYTHONUNBUFFERED=1 \
    RUSTEEZE_HOST=0.0.0.0 RUSTEEZE_PORT=8000 RUSTEEZE_CONFIG=/app/config.yaml HF_HOME=/data/huggingface
RUN apt-get update && apt-get install -y --no-install-recommends python3 curl && rm -rf /var/lib/apt/lists/*
COPY --from=build /opt/venv /opt/venv
WORKDIR /app
COPY --from=build /src/rusteeze_b200 ./rusteeze_b200
COPY config.example.yaml ./config.example.yaml
COPY config.example.yaml ./config.yaml
RUN useradd -r -u 1001 -m rusteeze && mkdir -p /data/huggingface && chown -R rusteeze /app /data
USER rusteeze
EXPOSE 8000
HEALTHCHECK --interval=30s --timeout=10s --start-period=300s --retries=3 \
    CMD curl -fsS http://localhost:${RUSTEEZE_PORT}/health/live || exit 1
ENTRYPOINT ["python", "-m", "rusteeze_b200"]
CMD ["serve"]
