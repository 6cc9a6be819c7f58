"""Host-side helpers on the CPU (no GPU): topology discovery over a fake sysfs tree, the
cpulist parser, the exclusive-core split, sg_compat::linear_to_sg_entries, and NUMA
binding of pool memory.  Compiled with g++ from tests/topology_probe.cpp.

Reference behaviour: include/gfd/pcie_topology.h:41-154 (discover_topology,
TopologyConfig::get_exclusive_cores), include/gfd/sg_task_queue.h:106-122
(linear_to_sg_entries), examples/05_multi_gpu_benchmark.cu:217-231 (pools bound to the
GPU's NUMA node)."""
import ctypes
import errno
import os
import subprocess
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_INC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
DEVICE_SG = np.dtype([("src", "<u8"), ("dst", "<u8"), ("size", "<u4"), ("tag", "<u4")])


@pytest.fixture(scope="module")
def lib():
    out = os.path.join(tempfile.mkdtemp(prefix="gfdtopo_"), "libgfdtopo.so")
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-Wall", "-Werror",
                           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "gfd_b200", "csrc"),
                           "-I", CUDA_INC, os.path.join(ROOT, "tests", "topology_probe.cpp"), "-o", out])
    l = ctypes.CDLL(out)
    vp, ip = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)
    l.probe_parse_list.argtypes = [ctypes.c_char_p, vp, ctypes.c_int]
    l.probe_parse_list.restype = ctypes.c_int
    l.probe_topology.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, vp, vp]
    l.probe_topology.restype = None
    l.probe_linear_to_sg.argtypes = [vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                     ctypes.c_uint32, ctypes.c_uint32]
    l.probe_linear_to_sg.restype = None
    l.probe_map_pool.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64),
                                 ip, ip]
    l.probe_map_pool.restype = ctypes.c_int
    l.probe_page_node.argtypes = [vp]
    l.probe_page_node.restype = ctypes.c_int
    l.probe_unmap_pool.argtypes = [vp, ctypes.c_uint64]
    l.probe_unmap_pool.restype = None
    return l


def parse(lib, s):
    out = np.zeros(64, np.int32)
    n = lib.probe_parse_list(s.encode(), out.ctypes.data, 32)
    return [tuple(out[2 * i:2 * i + 2].tolist()) for i in range(n)]


@pytest.mark.parametrize("text,want", [
    ("0-15", [(0, 15)]),
    ("0-31,64-95", [(0, 31), (64, 95)]),
    ("3", [(3, 3)]),
    ("0-3,8,10-11", [(0, 3), (8, 8), (10, 11)]),
    ("", []),
    ("7,", [(7, 7)]),
])
def test_cpulist_parser(lib, text, want):
    assert parse(lib, text) == want


def fake_sysfs(root, online, cpulists, gpu_nodes):
    """A sysfs tree: node/online, node/node<n>/cpulist, and one PCI device per GPU with
    its numa_node (None: the file is absent)."""
    nd = os.path.join(root, "devices", "system", "node")
    os.makedirs(nd)
    with open(os.path.join(nd, "online"), "w") as f:
        f.write(online + "\n")
    for n, cl in enumerate(cpulists):
        os.makedirs(os.path.join(nd, f"node{n}"))
        with open(os.path.join(nd, f"node{n}", "cpulist"), "w") as f:
            f.write(cl + "\n")
    ids = []
    for g, node in enumerate(gpu_nodes):
        bus = f"0000:{0x1b + 0x10 * g:02x}:00.0"
        d = os.path.join(root, "bus", "pci", "devices", bus)
        os.makedirs(d)
        if node is not None:
            with open(os.path.join(d, "numa_node"), "w") as f:
                f.write(f"{node}\n")
        ids.append(bus.upper())  # the CUDA runtime reports upper-case hex; sysfs names are lower case
    return ids


def topology(lib, root, ids):
    head = np.zeros(4, np.int32)
    out = np.zeros(8 * max(len(ids), 1), np.int32)
    blob = b"".join(i.encode() + b"\0" for i in ids)
    lib.probe_topology(root.encode(), blob, len(ids), head.ctypes.data, out.ctypes.data)
    keys = ("numa", "cpu_start", "cpu_end", "ht_offset", "cores", "excl_base", "excl_count", "bus")
    return head.tolist(), [dict(zip(keys, out[8 * g:8 * g + 8].tolist())) for g in range(len(ids))]


def test_two_nodes_with_hyperthreads_match_the_reference_layout(lib, tmp_path):
    ids = fake_sysfs(str(tmp_path), "0-1", ["0-31,64-95", "32-63,96-127"], [0, 0, 0, 0, 1, 1, 1, 1])
    head, gpus = topology(lib, str(tmp_path), ids)
    assert head == [2, 64, 32, 4]
    for g, t in enumerate(gpus):
        node = 0 if g < 4 else 1
        # the reference's formulas for this host shape (pcie_topology.h:80-131, :41-60):
        # cpu_start = node * cores, ht_offset = second range - first, cores / GPUs on the node
        assert t["numa"] == node
        assert (t["cpu_start"], t["cpu_end"], t["ht_offset"], t["cores"]) == (32 * node, 32 * node + 31, 64, 32)
        assert (t["excl_base"], t["excl_count"]) == (32 * node + 8 * (g % 4), 8)
        assert t["bus"] == 0x1b + 0x10 * g


def test_single_range_node_without_hyperthreads(lib, tmp_path):
    ids = fake_sysfs(str(tmp_path), "0", ["0-31"], [0, 0, 0])
    head, gpus = topology(lib, str(tmp_path), ids)
    assert head == [1, 32, 32, 3]
    assert [(t["excl_base"], t["excl_count"]) for t in gpus] == [(0, 10), (10, 10), (20, 10)]
    assert all(t["ht_offset"] == 0 and t["cores"] == 32 for t in gpus)


def test_single_core_node(lib, tmp_path):
    ids = fake_sysfs(str(tmp_path), "0", ["3"], [0, 0])
    head, gpus = topology(lib, str(tmp_path), ids)
    assert head == [1, 1, 1, 2]
    for t in gpus:
        assert (t["cpu_start"], t["cpu_end"], t["cores"]) == (3, 3, 1)
        assert (t["excl_base"], t["excl_count"]) == (3, 1)  # never zero cores


def test_gpu_without_node_maps_to_node_zero(lib, tmp_path):
    # numa_node -1 (a VM), no numa_node file, an unknown bus id, a node the host does not have
    ids = fake_sysfs(str(tmp_path), "0-1", ["0-15", "16-31"], [-1, None, 1, 5])
    ids[2] = ""
    head, gpus = topology(lib, str(tmp_path), ids)
    assert head[0] == 2
    assert [t["numa"] for t in gpus] == [0, 0, 0, 0]
    assert all((t["cpu_start"], t["cpu_end"]) == (0, 15) for t in gpus)
    assert [t["excl_count"] for t in gpus] == [4, 4, 4, 4]


def test_gpu_on_second_node_with_sparse_cpulist(lib, tmp_path):
    ids = fake_sysfs(str(tmp_path), "0-1", ["0-7", "8-11,40-43"], [1, 1])
    head, gpus = topology(lib, str(tmp_path), ids)
    assert [t["numa"] for t in gpus] == [1, 1]
    assert [(t["cpu_start"], t["cpu_end"], t["ht_offset"]) for t in gpus] == [(8, 11, 32)] * 2
    # physical cores per node come from node 0 (8): 4 per GPU.  The second GPU's share
    # starts past the node's first range; it gets the node's first core rather than none
    assert [(t["excl_base"], t["excl_count"]) for t in gpus] == [(8, 4), (8, 1)]


@pytest.mark.parametrize("start,count,size,tag", [(0, 1, 4096, 0), (5, 17, 512, 3), (1000, 64, 14336, 0xFFFFFFFF),
                                                   (0, 0, 4096, 1)])
def test_linear_to_sg_entries(lib, start, count, size, tag):
    cpu, gpu = 0x7f0000001000, 0x7e0000000000
    out = np.zeros(max(count, 1), DEVICE_SG)
    lib.probe_linear_to_sg(out.ctypes.data, cpu, gpu, size, start, count, tag)
    # reference semantics (sg_task_queue.h:106-122): entry i covers token start + i
    idx = np.arange(start, start + count, dtype=np.uint64) * np.uint64(size)
    assert np.array_equal(out["src"][:count], np.uint64(cpu) + idx)
    assert np.array_equal(out["dst"][:count], np.uint64(gpu) + idx)
    assert np.all(out["size"][:count] == size) and np.all(out["tag"][:count] == tag)
    if count == 0:
        assert not out.view(np.uint8).any()  # nothing written


def online_nodes():
    try:
        text = open("/sys/devices/system/node/online").read().strip()
    except OSError:
        return [0]
    nodes = []
    for part in text.split(","):
        if "-" in part:
            a, b = part.split("-")
            nodes += list(range(int(a), int(b) + 1))
        elif part:
            nodes.append(int(part))
    return nodes or [0]


def map_pool(lib, nbytes, node):
    p, ln, bound, err = ctypes.c_void_p(), ctypes.c_uint64(), ctypes.c_int(), ctypes.c_int()
    rc = lib.probe_map_pool(nbytes, node, ctypes.byref(p), ctypes.byref(ln), ctypes.byref(bound), ctypes.byref(err))
    return rc, p.value, ln.value, bound.value, err.value


@pytest.mark.parametrize("node", online_nodes())
def test_pool_pages_land_on_the_bound_node(lib, node):
    rc, p, ln, bound, err = map_pool(lib, 5 << 20, node)
    if rc != 0 and err in (errno.EPERM, errno.ENOSYS):
        pytest.skip("mbind is not permitted in this container")
    assert rc == 0 and bound == node and ln == 6 << 20
    try:
        for off in range(0, ln, 1 << 20):
            where = lib.probe_page_node(p + off)
            if where == -1:
                pytest.skip("get_mempolicy is not permitted in this container")
            assert where == node
    finally:
        lib.probe_unmap_pool(p, ln)


def test_pool_on_a_missing_node_is_refused(lib):
    missing = max(online_nodes()) + 1
    rc, p, ln, bound, err = map_pool(lib, 1 << 20, missing)
    assert rc == -1 and p is None and err != 0
    rc, p, ln, bound, err = map_pool(lib, 1 << 20, 64)  # beyond one node mask
    assert rc == -1 and err == errno.EINVAL


def test_unbound_pool(lib):
    rc, p, ln, bound, err = map_pool(lib, 1, -1)
    assert rc == 0 and bound == -1 and ln == 2 << 20
    lib.probe_unmap_pool(p, ln)


@pytest.mark.gpu
@pytest.mark.parametrize("node", online_nodes())
def test_gfd_pool_alloc_binds_and_reports_the_node(lib, gpu_ctx, node):
    """gfd_pool_alloc(numa_node=k): the pool reports node k and its pages sit on node k;
    a node the host does not have is refused."""
    import gfd_b200
    pool = gpu_ctx.pool(6 << 20, numa_node=node)
    try:
        assert pool.numa_node == node
        for off in range(0, 6 << 20, 1 << 20):
            where = lib.probe_page_node(pool.ptr + off)
            assert where in (node, -1)  # -1: get_mempolicy not permitted here
    finally:
        pool.free()
    with pytest.raises(gfd_b200.GfdError) as exc:
        gpu_ctx.pool(1 << 20, numa_node=max(online_nodes()) + 1)
    assert exc.value.code == gfd_b200.GFD_ERR_INVALID
    auto = gpu_ctx.pool(1 << 20)  # the GPU's own node when the host reports one, else unbound
    try:
        assert auto.numa_node in [-1] + online_nodes()
    finally:
        auto.free()
