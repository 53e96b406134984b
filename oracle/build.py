"""Build recipes for the CPU checkers (TEST INFRASTRUCTURE ONLY).

* ``build_oracle()`` compiles this directory's own C restatement
  (``mmnb_oracle.c``) into ``oracle/libmmnb_oracle.so``.
* ``build_reference()`` compiles the reference's own algorithm, taken from the
  xrGPU sources where they lie, into ``oracle/_ref/libmmnb_ref.so``. The GLSL
  helpers are plain C-like functions, so they compile as C++ once a prelude
  supplies the storage-access functions the shader framework would provide
  (``readU``/``readF``/``get``/``put``/``arg``/``has``/``size``), the same
  technique the reference's own host tests use for its GLSL helpers
  (``tests/test_native_half.py:20-33``, ``tests/test_extended_quant_cache.py:24-83``).
  Used files, relative to the xrGPU project root:

    - ``kernels/_shared/shaders/half.glsl`` (included whole), and
    - the ``nbitWeight``, ``packedInput`` and ``packedMatmul`` definitions of
      ``kernels/_shared/extended/shaders/complex_kernel.glsl`` (lines 80, 81, 83),
      selected by their signatures at build time.

  Nothing of the reference is copied into this repository: the generated
  translation unit lives in a temporary directory and only the shared object
  is written, under ``oracle/_ref/`` (git-ignored). It is built only where the
  reference checkout exists; elsewhere the prebuilt object is used.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libmmnb_oracle.so"
REF_DIR = HERE / "_ref"
REF_SO = REF_DIR / "libmmnb_ref.so"
DEFAULT_REFERENCE = Path(os.environ.get("XRGPU_REFERENCE_ROOT", "/root/reference"))

SIGNATURES = ("float nbitWeight(", "float packedInput(", "void packedMatmul(")

# Prelude: storage-access functions for opcode 1025's input slots
# (0 aT, 1 bT, 2 scalesT, 3 zeroPointsT, 4 biasT; complex_plan.cpp:34) over
# native-width host arrays. Bounds checks record code 1 like framework.glsl:44.
PRELUDE = r"""
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>
using uint = uint32_t;
static inline float uintBitsToFloat(uint x){float y;std::memcpy(&y,&x,4);return y;}
static inline uint floatBitsToUint(float x){uint y;std::memcpy(&y,&x,4);return y;}
#include "HALF_GLSL"
static const uint NONE = 0xffffffffu;
static const uint D_F32 = 0u, D_F16 = 1u, D_U8 = 6u;
struct Ctx {
  const void* in[5]; int dt[5]; uint64_t count[5];
  void* out; int out_dt; uint64_t out_count; int64_t out_ld, out_col0;
  uint args[128]; uint failure;
};
static thread_local Ctx* C = nullptr;
static inline uint op(){return 1025u;}
static inline uint arg(uint i){return C->args[i];}
static inline float argF(uint i){return uintBitsToFloat(C->args[i]);}
static inline bool has(uint s){return s<5u && C->in[s]!=nullptr;}
static inline uint size(uint s){return has(s)?uint(C->count[s]):0u;}
static inline void fail(uint code){C->failure=std::max(C->failure,code);}
static inline uint readU(uint s,uint i){
  if(!has(s)||i>=size(s)){fail(1u);return 0u;}
  if(C->dt[s]==int(D_F32))return ((const uint*)C->in[s])[i];
  if(C->dt[s]==int(D_F16))return ((const uint16_t*)C->in[s])[i];
  return ((const uint8_t*)C->in[s])[i];
}
static inline float readF(uint s,uint i){uint v=readU(s,i);int t=C->dt[s];if(t==int(D_F32))return uintBitsToFloat(v);if(t==int(D_F16))return xrgpuHalfToFloat(v);return float(v);}
static inline float get(uint s,uint i,float fallback){return s!=NONE&&has(s)&&i<size(s)?readF(s,i):fallback;}
static inline void put(uint canonical,uint i,float x){
  if(canonical!=0u||i>=C->out_count)return;
  uint n=C->args[2];uint row=i/n,col=i%n;int64_t o=int64_t(row)*C->out_ld+C->out_col0+col;
  if(C->out_dt==int(D_F32))((float*)C->out)[o]=x;else ((uint16_t*)C->out)[o]=uint16_t(xrgpuFloatToHalf(x));
}
static inline float inversesqrt(float x){return 1.0f/std::sqrt(x);}
static inline float fused(float x,uint){return x;}        // not reached by opcode 1025
static inline float bnbWeight(uint,uint){return 0.0f;}     // not reached by opcode 1025
"""

EPILOGUE = r"""
extern "C" uint mmnb_ref_half_to_float_bits(uint h){return floatBitsToUint(xrgpuHalfToFloat(h));}
extern "C" uint mmnb_ref_float_bits_to_half(uint f){return xrgpuFloatToHalf(uintBitsToFloat(f));}
static uint64_t elem_bytes(int dt){return dt==int(D_F32)?4:dt==int(D_F16)?2:1;}
// Reference packedMatmul over output columns [col0, col1), split across threads by
// column range (each thread sees its own column slice as a complete problem).
extern "C" int mmnb_ref_matmul(const void* a,int a_dt,int64_t rows,int64_t K,int64_t N,
    const uint8_t* b,const void* scales,const void* zp,int zp_dt,const void* bias,
    int64_t block_size,int64_t bits,void* y,int64_t col0,int64_t col1,int threads){
  if(col0<0||col1>N||col1<col0)return 100;
  int64_t blocks=(K+block_size-1)/block_size,blob=(block_size*bits+7)/8,span=col1-col0;
  if(threads<1)threads=1;if(threads>256)threads=256;if(span<threads)threads=span>0?int(span):1;
  std::vector<Ctx> ctx(threads);std::vector<std::thread> pool;
  for(int t=0;t<threads;++t){
    int64_t c0=col0+span*t/threads,c1=col0+span*(t+1)/threads,w=c1-c0;Ctx& c=ctx[t];std::memset(&c,0,sizeof(Ctx));
    c.in[0]=a;c.dt[0]=a_dt;c.count[0]=uint64_t(rows*K);
    c.in[1]=b+c0*blocks*blob;c.dt[1]=int(D_U8);c.count[1]=uint64_t(w*blocks*blob);
    c.in[2]=(const char*)scales+c0*blocks*elem_bytes(a_dt);c.dt[2]=a_dt;c.count[2]=uint64_t(w*blocks);
    c.in[3]=zp?(const void*)((const char*)zp+c0*blocks*elem_bytes(zp_dt)):nullptr;c.dt[3]=zp_dt;c.count[3]=zp?uint64_t(w*blocks):0;
    c.in[4]=bias?(const void*)((const char*)bias+c0*elem_bytes(a_dt)):nullptr;c.dt[4]=a_dt;c.count[4]=bias?uint64_t(w):0;
    c.out=y;c.out_dt=a_dt;c.out_count=uint64_t(rows*w);c.out_ld=N;c.out_col0=c0;
    c.args[0]=1025u;c.args[1]=uint(K);c.args[2]=uint(w);c.args[3]=uint(block_size);c.args[4]=uint(bits);c.args[5]=1u;c.args[6]=1u;c.args[7]=floatBitsToUint(1e-5f);
  }
  auto work=[&](int t){C=&ctx[t];if(ctx[t].args[2])packedMatmul();C=nullptr;};
  for(int t=1;t<threads;++t)pool.emplace_back(work,t);
  work(0);for(auto& th:pool)th.join();
  uint failure=0;for(auto& c:ctx)failure=std::max(failure,c.failure);return int(failure);
}
"""


def _compiler(name: str) -> str:
    found = shutil.which(name)
    if not found:
        raise RuntimeError(f"{name} is required to build the CPU checkers")
    return found


def build_oracle(force: bool = False) -> Path:
    """Compile ``mmnb_oracle.c`` (own restatement) into ``libmmnb_oracle.so``."""
    src = HERE / "mmnb_oracle.c"
    if not force and ORACLE_SO.exists() and ORACLE_SO.stat().st_mtime >= src.stat().st_mtime:
        return ORACLE_SO
    tmp = ORACLE_SO.with_suffix(".so.tmp")
    subprocess.run([_compiler("gcc"), "-O2", "-std=c11", "-ffp-contract=off", "-fPIC", "-shared",
                    "-pthread", str(src), "-o", str(tmp), "-lm"], check=True)
    os.replace(tmp, ORACLE_SO)
    return ORACLE_SO


def extract_reference_functions(reference_root: Path) -> str:
    """Return the three opcode-1025 function definitions from complex_kernel.glsl."""
    path = reference_root / "kernels/_shared/extended/shaders/complex_kernel.glsl"
    found = {}
    for line in path.read_text().splitlines():
        for sig in SIGNATURES:
            if line.startswith(sig):
                found[sig] = line
    missing = [s for s in SIGNATURES if s not in found]
    if missing:
        raise RuntimeError(f"reference functions not found: {missing}")
    return "\n".join(found[s] for s in SIGNATURES)


def build_reference(reference_root: Path | None = None, force: bool = False) -> Path | None:
    """Compile the reference's own algorithm into ``oracle/_ref/libmmnb_ref.so``.

    Returns ``None`` when the reference checkout is absent (e.g. on a GPU box,
    which uses the prebuilt object shipped with the working tree).
    """
    root = Path(reference_root) if reference_root else DEFAULT_REFERENCE
    half = root / "kernels/_shared/shaders/half.glsl"
    if not half.exists():
        return REF_SO if REF_SO.exists() else None
    if REF_SO.exists() and not force:
        return REF_SO
    REF_DIR.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmpdir:
        src = Path(tmpdir) / "mmnb_ref.cpp"
        src.write_text(PRELUDE.replace("HALF_GLSL", str(half)) + "\n"
                       + extract_reference_functions(root) + "\n" + EPILOGUE)
        tmp = REF_SO.with_suffix(".so.tmp")
        subprocess.run([_compiler("g++"), "-O2", "-std=c++17", "-ffp-contract=off", "-fPIC",
                        "-shared", "-pthread", str(src), "-o", str(tmp)], check=True)
        os.replace(tmp, REF_SO)
    return REF_SO


if __name__ == "__main__":
    print(build_oracle(force=True))
    print(build_reference(force=True))
