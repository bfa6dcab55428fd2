"""One launch of each hot-path kernel (KDA prefill, indexer logits, canonical top-k, expansion, sparse MLA, mHC) at a
small size whose inputs exceed L2: the program the ncu summaries of these kernels are captured from."""
import sys, ctypes, numpy as np, torch
sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parent.parent))
import __graft_entry__ as g; g.import_package()
from ssengine_b200 import indexer, mla, lib
from ssengine_b200.kda import KdaLayer, seq_table
dev = torch.device("cuda:0")
gen = torch.Generator(device=dev).manual_seed(1)
rnd = lambda *s: torch.randn(*s, device=dev, generator=gen)
# KDA: 32 heads, 8192 tokens, 4 requests
H, P, T = 32, 4096, 8192
lens = [3000, 2500, 1700, 992]; st = np.concatenate([[0], np.cumsum(lens)])
x = rnd(T, 3 * P).to(torch.bfloat16); gg = rnd(T, P).to(torch.bfloat16); be = rnd(T, H).to(torch.bfloat16)
L = KdaLayer((torch.rand(3 * P, 4, device=dev) - 0.5).to(torch.bfloat16), torch.rand(H, device=dev) * 2 - 1, rnd(P) * 0.5)
cst = rnd(5, 3, 3 * P).to(torch.bfloat16); rst = rnd(5, H, 128, 128) * 0.05; o = torch.empty(T, P, dtype=torch.bfloat16, device=dev)
L.prefill(x, gg, be, o, seq_table([(int(st[i]), int(st[i + 1]), i + 1, 1) for i in range(4)], dev), cst, rst)
torch.cuda.synchronize(); del x, gg, o
# DSA: 4096 rows of 2 requests with 16k prefixes
R, lens, prefix = 2, np.array([2048, 2048]), np.array([16384, 8192])
T = int(lens.sum()); qsl = np.array([0, 2048, 4096], np.int32)
positions = np.concatenate([np.arange(p, p + n) for p, n in zip(prefix, lens)]).astype(np.int64)
npg = [-(-(int(p) + int(n)) // 128) for p, n in zip(prefix, lens)]; width = max(npg)
table = np.full((R, width), -1, np.int32); at = 1
for r, n in enumerate(npg): table[r, :n] = np.arange(at, at + n); at += n
pos = torch.from_numpy(positions).to(dev); tab = torch.from_numpy(table).to(dev)
groups = torch.from_numpy(indexer.work_groups(qsl[:-1], lens, prefix)).to(dev)
q = rnd(T, 32, 128).to(torch.bfloat16); w = torch.rand(T, 32, device=dev); kp = rnd(at * 32, 128).to(torch.bfloat16)
ldl = int(((positions.max() + 1) // 4 + 127) // 128 * 128); lg = torch.empty(T, ldl, device=dev)
indexer.logits(q, w, kp, tab, groups, lg)
ids = torch.empty(T, 512, dtype=torch.int32, device=dev); indexer.topk(lg, pos, 512, ids)
tok = torch.empty(T, 2056, dtype=torch.int32, device=dev); indexer.expand(ids, pos, tok)
qm = (rnd(T, 64, 576) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
kv = rnd(at * 128, 576).to(torch.float8_e4m3fn).view(torch.uint8)
mo = torch.empty(T, 64, 512, dtype=torch.bfloat16, device=dev)
mla.sparse_mla(qm, kv, tok, torch.from_numpy(qsl).to(dev), tab, 192 ** -0.5, mo, n_idx=2051)
torch.cuda.synchronize(); del qm, kv, mo, lg
# mHC at T = 8192, H = 4096
Tm, Hm = 8192, 4096
xm = rnd(Tm, Hm).to(torch.bfloat16); res = rnd(Tm, 4, Hm).to(torch.bfloat16)
pin = torch.rand(Tm, 4, device=dev) + 0.5; cin = torch.softmax(rnd(Tm, 4, 4), 1)
fn = rnd(24, 4 * Hm) / 128; sc = torch.tensor([0.8, 0.6, 1.5], device=dev); base = rnd(24) * 0.3
nw = torch.ones(Hm, device=dev).to(torch.bfloat16); nr = torch.empty_like(res); po = torch.empty(Tm, 4, device=dev)
co = torch.empty(Tm, 4, 4, device=dev); y = torch.empty_like(xm)
prm = lib.MhcParamsC(Hm, 4, fn.data_ptr(), sc.data_ptr(), base.data_ptr(), nw.data_ptr(), 1e-6, 1e-2, 1e-6, 2.0, 1e-6, 20)
so = lib.load(); ws = torch.empty(int(so.ssb_mhc_workspace_bytes(Tm)), dtype=torch.uint8, device=dev)
lib.check("mhc", so.ssb_mhc_ws(ctypes.byref(prm), xm.data_ptr(), res.data_ptr(), pin.data_ptr(), cin.data_ptr(),
          nr.data_ptr(), po.data_ptr(), co.data_ptr(), y.data_ptr(), Tm, ws.data_ptr(), ws.numel(),
          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
torch.cuda.synchronize()
print("ok")
