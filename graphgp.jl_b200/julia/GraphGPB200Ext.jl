module GraphGPB200Ext

# Thin ccall layer over libgraphgp_b200.so for CuArray-backed GraphGPProblems: the drop-in
# replacement of GraphGP.jl's KernelAbstractions launches and of ext/GraphGPCUDAExt.jl.  Load it
# with `using GraphGP, CUDA` plus this extension (see INTEGRATION.md); the library is found at
# ENV["GRAPHGP_B200_LIB"], as ext/GraphGPCUDAExt.jl:15-24 finds libgraphgpcapi.so.
#
# Each GraphGPProblem gets one library handle (device copies of int32 neighbours, padded coords
# and the interpolation table), cached in a WeakKeyDict and freed by a finalizer.  Arrays are
# passed in GraphGP.jl's own layout: coords (D,N) UInt32, neighbors (K,M) Int 1-based, offsets
# and indices on the host.  Every call is ordered on CUDA.jl's task-local stream.

using GraphGP
using CUDA
using Libdl
import GraphGP: GraphGPProblem, npoints, nrefined, nneighbors, ndims_space, nbins

const LIBREF = Ref{Ptr{Cvoid}}(C_NULL)
function _lib()
    LIBREF[] != C_NULL && return LIBREF[]
    path = get(ENV, "GRAPHGP_B200_LIB", joinpath(@__DIR__, "..", "libgraphgp_b200.so"))
    isfile(path) || error("libgraphgp_b200.so not found at $path (set GRAPHGP_B200_LIB)")
    LIBREF[] = Libdl.dlopen(path)
    return LIBREF[]
end
_sym(name::Symbol) = Libdl.dlsym(_lib(), name)
_stream() = reinterpret(Ptr{Cvoid}, CUDA.stream().handle)

function _check(rc, what)
    rc == 0 && return nothing
    msg = unsafe_string(ccall(_sym(:gpb2_last_error), Cstring, ()))
    rc == 8 && throw(ArgumentError("$what: $msg"))          # check_graph invariant
    error("$what returned $rc: $msg")
end

const HANDLES = WeakKeyDict{GraphGPProblem, Ptr{Cvoid}}()

function _handle(prob::GraphGPProblem{T}) where {T}
    h = get(HANDLES, prob, C_NULL)
    h != C_NULL && return h
    prob.coords isa CuArray || error("GraphGPB200Ext needs a CuArray problem (to_backend)")
    dtype = T === Float32 ? Cint(0) : T === Float64 ? Cint(1) : error("Float32/Float64 only")
    nb = prob.neighbors
    offs = Vector{Int64}(prob.offsets)
    idxv = prob.indices === nothing ? nothing : Vector{Int64}(prob.indices)
    out = Ref{Ptr{Cvoid}}(C_NULL)
    GC.@preserve offs idxv begin
        rc = ccall(_sym(:gpb2_problem_create), Cint,
            (Ptr{Ptr{Cvoid}}, Cint, Cint, CuPtr{UInt32}, Int64, Int64, CuPtr{Cvoid}, Cint, Cint,
             Int64, Ptr{Int64}, Int64, Int64, Cdouble, CuPtr{Cvoid}, CuPtr{Cvoid}, Int64,
             Ptr{Int64}, Cint, Ptr{Cvoid}),
            out, dtype, CUDA.deviceid(CUDA.device()), prob.coords, ndims_space(prob),
            npoints(prob), reinterpret(CuPtr{Cvoid}, pointer(nb)), Cint(sizeof(eltype(nb))),
            Cint(1), nneighbors(prob), offs, length(offs), prob.n0, Float64(prob.scale),
            reinterpret(CuPtr{Cvoid}, pointer(prob.bins)),
            reinterpret(CuPtr{Cvoid}, pointer(prob.vals)), nbins(prob),
            idxv === nothing ? Ptr{Int64}(C_NULL) : pointer(idxv), Cint(1), _stream())
        _check(rc, "gpb2_problem_create")
    end
    HANDLES[prob] = out[]
    finalizer(prob) do _
        ccall(_sym(:gpb2_problem_destroy), Cint, (Ptr{Cvoid},), out[])
    end
    return out[]
end

_ptr(x::CuArray) = reinterpret(CuPtr{Cvoid}, pointer(x))

# --- refine layer (replaces the launches of src/api.jl:52-55, 87-90, 126-138) -----------------
function refine_b200!(values::CuArray{T}, prob::GraphGPProblem{T}, xi::CuArray{T}) where {T}
    _check(ccall(_sym(:gpb2_refine), Cint, (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
        _handle(prob), _ptr(values), _ptr(xi), _stream()), "gpb2_refine")
    return values
end

function refine_inv_b200!(xi::CuArray{T}, prob::GraphGPProblem{T}, values::CuArray{T}) where {T}
    _check(ccall(_sym(:gpb2_refine_inv), Cint, (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
        _handle(prob), _ptr(values), _ptr(xi), _stream()), "gpb2_refine_inv")
    return xi
end

function refine_logdet_b200(prob::GraphGPProblem)
    out = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_refine_logdet), Cint, (Ptr{Cvoid}, Ref{Cdouble}, Ptr{Cvoid}),
        _handle(prob), out, _stream()), "gpb2_refine_logdet")
    return out[]
end

# --- orchestrated operations, ORIGINAL order (src/orchestrate.jl, src/grad*.jl) --------------
function generate_b200(prob::GraphGPProblem{T}, xi::CuArray{T}) where {T}
    out = similar(xi)
    _check(ccall(_sym(:gpb2_generate), Cint, (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
        _handle(prob), _ptr(xi), _ptr(out), _stream()), "gpb2_generate")
    return out
end

function generate_inv_b200(prob::GraphGPProblem{T}, values::CuArray{T}) where {T}
    out = similar(values)
    _check(ccall(_sym(:gpb2_generate_inv), Cint,
        (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
        _handle(prob), _ptr(values), _ptr(out), _stream()), "gpb2_generate_inv")
    return out
end

function generate_logdet_b200(prob::GraphGPProblem{T}) where {T}
    out = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_generate_logdet), Cint, (Ptr{Cvoid}, Ref{Cdouble}, Ptr{Cvoid}),
        _handle(prob), out, _stream()), "gpb2_generate_logdet")
    return T(out[])
end

function generate_grad_xi_b200(prob::GraphGPProblem{T}, vbar::CuArray{T}) where {T}
    out = similar(vbar)
    _check(ccall(_sym(:gpb2_generate_grad_xi), Cint,
        (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
        _handle(prob), _ptr(vbar), _ptr(out), _stream()), "gpb2_generate_grad_xi")
    return out
end

function generate_grad_vals_b200(prob::GraphGPProblem{T}, xi::CuArray{T}, vbar::CuArray{T}) where {T}
    out = CUDA.zeros(T, nbins(prob))
    _check(ccall(_sym(:gpb2_generate_grad_vals), Cint,
        (Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
        _handle(prob), _ptr(xi), _ptr(vbar), _ptr(out), _stream()), "gpb2_generate_grad_vals")
    return out
end

function refine_logdet_grad_vals_b200(prob::GraphGPProblem{T}) where {T}
    out = CUDA.zeros(T, nbins(prob))
    _check(ccall(_sym(:gpb2_refine_logdet_grad_vals), Cint,
        (Ptr{Cvoid}, CuPtr{Cvoid}, Ptr{Cdouble}, Ptr{Cvoid}),
        _handle(prob), _ptr(out), C_NULL, _stream()), "gpb2_refine_logdet_grad_vals")
    return out
end

end # module
