"""CPU-only checks of the C ABI: the library loads, exports every function include/k3c.h
declares, and the ctypes mirrors of the header's structs have the C layout."""
import ctypes as C
import os
import re
import subprocess
import tempfile

from conftest import ROOT

HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:extern\s+)?[A-Za-z_][\w\s\*]*?\b(k3c?_\w+)\s*\(", src, re.M):
            names.add(m.group(1))
    return names


def test_header_declares_dropin_and_device_api():
    names = declared_functions()
    for n in ("k3_mxfp4_dequant", "k3_matmul_mxfp4", "k3_matmul_q8", "k3_router",
              "k3c_mxfp4_gemv", "k3c_moe_decode", "k3c_router_select", "k3c_last_error"):
        assert n in names, n


def test_library_exports_every_declared_symbol(k3):
    L = k3.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(L, n)]
    assert not missing, missing
    assert hasattr(L, "k3_expert_drops")       # extern long, include/k3c.h
    assert C.c_long.in_dll(L, "k3_expert_drops").value == 0
    assert L.k3c_version().decode().endswith("sm_100a")


def test_library_built_for_sm100a_only():
    mk = open(os.path.join(ROOT, "kimi-k3-in-rust_b200", "csrc", "Makefile")).read()
    arch = re.search(r"^ARCH\s*:=\s*(.*)$", mk, re.M).group(1).split()
    assert arch == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "use_fast_math" not in mk.split("NVFLAGS")[1].split("\n")[0]


def test_struct_layouts_match_header(k3):
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "k3c.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu\n", sizeof(K3ExpertQ), offsetof(K3ExpertQ, p2),
         sizeof(k3c_moe_layer), offsetof(k3c_moe_layer, router_w), offsetof(k3c_moe_layer, shared));
  return 0; }
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        got = [int(v) for v in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    want = [C.sizeof(k3.K3ExpertQ), k3.K3ExpertQ.p2.offset, C.sizeof(k3.MoeLayerC),
            k3.MoeLayerC.router_w.offset, k3.MoeLayerC.shared.offset]
    assert got == want


def test_errors_are_reported_without_a_gpu(k3):
    """Argument validation runs before any CUDA call, so it is testable here."""
    L = k3.lib()
    rc = L.k3c_mxfp4_gemv(None, 4, None, 4, 1, None, None, 7, 4, 32, None)   # odd `in`
    assert rc == -1 and b"odd" in L.k3c_last_error()
    rc = L.k3c_mxfp4_gemv(None, 4, None, 64, 1, None, None, 64, 4, 65, None)  # group > 64
    assert rc == -1 and b"group" in L.k3c_last_error()


def test_pool_and_ep_struct_layouts_match_header(k3):
    """The ctypes mirrors of the tensor-core layer, the expert-parallel peer table and the IPC
    handle have the C layout (offsets of every pointer array)."""
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "k3c.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\n",
         sizeof(k3c_moe_pool_layer), offsetof(k3c_moe_pool_layer, run_of),
         offsetof(k3c_moe_pool_layer, shared_run), offsetof(k3c_moe_pool_layer, terms),
         sizeof(k3c_ep_peers), offsetof(k3c_ep_peers, ntok), offsetof(k3c_ep_peers, x),
         offsetof(k3c_ep_peers, idx), offsetof(k3c_ep_peers, wt), offsetof(k3c_ep_peers, recv),
         offsetof(k3c_ep_peers, local_only), offsetof(k3c_ep_peers, x_ready), sizeof(k3c_ipc_handle));
  return 0; }
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        got = [int(v) for v in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    P, E = k3.MoePoolLayerC, k3.EpPeersC
    want = [C.sizeof(P), P.run_of.offset, P.shared_run.offset, P.terms.offset,
            C.sizeof(E), E.ntok.offset, E.x.offset, E.idx.offset, E.wt.offset, E.recv.offset,
            E.local_only.offset, E.x_ready.offset, C.sizeof(k3.IpcHandleC)]
    assert got == want


def test_ep_arguments_are_checked_without_a_gpu(k3):
    """The expert-parallel entry points validate the peer table before any CUDA call."""
    L = k3.lib()
    peers = k3.EpPeersC()
    peers.world, peers.rank, peers.t_max = 9, 0, 16                 # more ranks than supported
    layer = k3.MoePoolLayerC()
    layer.hidden, layer.inter, layer.n_experts, layer.topk = 512, 256, 8, 2
    assert L.k3c_moe_prefill_ep_scratch(C.byref(layer), C.byref(peers)) == 0
    rc = L.k3c_moe_prefill_ep_experts(C.byref(layer), C.byref(peers), None, 0, None)
    assert rc == -1 and b"peers" in L.k3c_last_error()
    peers.world = 2                                                   # buffers missing
    rc = L.k3c_moe_prefill_ep_experts(C.byref(layer), C.byref(peers), None, 0, None)
    assert rc == -1 and b"buffers" in L.k3c_last_error()
    rc = L.k3c_moe_ep_combine(None, C.byref(peers), 512, 2, None, 8, 1, None)
    assert rc == -1


def test_latent_struct_layout_and_argument_checks(k3):
    """The latent layer's ctypes mirror has the C layout, and the latent entry points reject
    bad arguments before any CUDA call."""
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "k3c.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\n", sizeof(k3c_moe_latent_layer),
         offsetof(k3c_moe_latent_layer, experts), offsetof(k3c_moe_latent_layer, router_w),
         offsetof(k3c_moe_latent_layer, latent_norm), offsetof(k3c_moe_latent_layer, wdt),
         offsetof(k3c_moe_latent_layer, situ_b2));
  return 0; }
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        got = [int(v) for v in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    M = k3.MoeLatentLayerC
    assert got == [C.sizeof(M), M.experts.offset, M.router_w.offset, M.latent_norm.offset,
                   M.wdt.offset, M.situ_b2.offset]

    L = k3.lib()
    lay = M()
    lay.hidden, lay.wdt, lay.n_shared, lay.latent_norm_on = 256, 1, 2, 1
    lay.situ_b1, lay.situ_b2, lay.rms_eps = 4.0, 25.0, 1e-5
    ex = lay.experts
    ex.hidden, ex.inter, ex.n_experts, ex.topk, ex.act, ex.terms, ex.shared_run = 128, 128, 8, 2, 1, 3, -1
    dummy = 4096
    lay.router_w = lay.down = lay.up = lay.sh1 = lay.sh3 = lay.sh2 = lay.latent_norm = dummy
    rc = L.k3c_moe_latent_decode(None, None, 70000, C.byref(lay), None, None, None, None, 0, None)
    assert rc == -1 and b"ntok" in L.k3c_last_error()
    lay.wdt = 3
    rc = L.k3c_moe_latent_decode(None, None, 4, C.byref(lay), None, None, None, None, 0, None)
    assert rc == -1 and b"wdt" in L.k3c_last_error()
    lay.wdt, ex.shared_run = 1, 0
    lay.experts = ex
    rc = L.k3c_moe_latent_decode(None, None, 4, C.byref(lay), None, None, None, None, 0, None)
    assert rc == -1 and b"shared_run" in L.k3c_last_error()
    ex.shared_run = -1
    lay.experts, lay.situ_b1 = ex, 3.0
    rc = L.k3c_moe_latent_decode(None, None, 4, C.byref(lay), None, None, None, None, 0, None)
    assert rc == -1 and b"SiTU" in L.k3c_last_error()
    lay.situ_b1, lay.sh2 = 4.0, None
    rc = L.k3c_moe_latent_decode(None, None, 4, C.byref(lay), None, None, None, None, 0, None)
    assert rc == -1 and b"missing" in L.k3c_last_error()
    assert L.k3c_mmw(None, 8, None, 8, 33, None, 1, 8, 8, 0, None) == -1
    assert L.k3c_mmw(dummy, 8, dummy, 8, 2, dummy, 2, 8, 8, 0, None) == -1
    assert b"int8" in L.k3c_last_error()


REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def test_reference_types_have_the_reference_layout(k3):
    """K3ExpertQ, K3ExpertSrc, K3Cfg and K3MoeW as include/k3c.h mirrors them have the
    offsets and sizes of the reference's include/k3/k3.h (oracle/_ref/abi_ref, built against
    the reference's header), and the ctypes mirrors have the same."""
    ref_exe = os.path.join(REF_DIR, "abi_ref")
    if not os.path.exists(ref_exe):
        import pytest
        pytest.skip("oracle/_ref/abi_ref not built (needs the reference tree)")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "abi_ours")
        subprocess.run(["gcc", "-O1", "-std=gnu99", "-DUSE_K3C", "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "oracle", "abi_layout.c"), "-o", exe], check=True)
        ours = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    ref = subprocess.run([ref_exe], capture_output=True, text=True, check=True).stdout
    assert ours == ref
    lay = {}
    for line in ref.splitlines():
        parts = line.split()
        if "." in parts[0] and len(parts) == 3:
            lay[parts[0]] = int(parts[1])
        elif len(parts) == 2 and parts[1].isdigit():
            lay[parts[0]] = int(parts[1])
    for cname, ct in (("K3Cfg", k3.K3CfgC), ("K3MoeW", k3.K3MoeWC), ("K3ExpertSrc", k3.K3ExpertSrcC),
                      ("K3ExpertQ", k3.K3ExpertQ)):
        assert C.sizeof(ct) == lay[cname], cname
        for f, _ in ct._fields_:
            assert getattr(ct, f).offset == lay[f"{cname}.{f}"], (cname, f)


def test_k3_moe_scratch_is_the_references(k3, ora):
    """k3_moe_scratch (no GPU needed) returns the reference's float count, so callers size
    their scratch exactly as before."""
    if not ora.ref_available():
        import pytest
        pytest.skip("oracle/_ref not built")
    R = ora.ref()
    R.k3_moe_scratch.restype = C.c_size_t
    R.k3_moe_scratch.argtypes = [C.c_void_p]
    for hidden, latent, inter, n_shared in ((128, 64, 48, 2), (7168, 3584, 3072, 2), (512, 256, 256, 0)):
        c = k3.K3CfgC()
        c.hidden, c.latent, c.moe_inter, c.n_shared = hidden, latent, inter, n_shared
        assert k3.lib().k3_moe_scratch(C.byref(c)) == R.k3_moe_scratch(C.addressof(c))


def test_reference_programs_bind_to_the_library():
    """The reference's own test_ops and bench_kernels built against libk3cuda.so
    (oracle/Makefile): every k3_* entry point the library defines resolves to it, both from the
    test program and from the reference's k3_ops.c (interposition), checked by the dynamic
    linker with all bindings resolved at start-up."""
    exe = os.path.join(REF_DIR, "test_ops_gpu")
    if not os.path.exists(exe):
        import pytest
        pytest.skip("oracle/_ref/test_ops_gpu not built")
    env = dict(os.environ, LD_BIND_NOW="1", LD_DEBUG="bindings")
    r = subprocess.run([exe, "/nonexistent"], capture_output=True, text=True, env=env, timeout=120)
    bind = {}
    for line in r.stderr.splitlines():
        m = re.search(r"binding file (\S+) \[0\] to (\S+) \[0\]: normal symbol `(k3_\w+)'", line)
        if m:
            bind[(os.path.basename(m.group(1)), m.group(3))] = os.path.basename(m.group(2))
    for sym in ("k3_moe", "k3_router", "k3_matmul", "k3_matmul_bf16", "k3_mxfp4_dequant", "k3_moe_scratch"):
        assert bind.get(("test_ops_gpu", sym)) == "libk3cuda.so", sym
    for sym in ("k3_moe", "k3_moe_prefill", "k3_router", "k3_matmul", "k3_matmul_bf16", "k3_matmul_mxfp4",
                "k3_matmul_q8", "k3_expert_drops"):
        assert bind.get(("libk3ops.so", sym)) == "libk3cuda.so", sym
    assert bind.get(("libk3ops.so", "k3_rmsnorm")) == "libk3ops.so"   # the rest stays the reference's
